/* TEST INFRASTRUCTURE ONLY: adapter that serves the hook-patched forward
 * pass's attention block with the B200 shim through the integration glue
 * (lestramanika_b200/hook/pickle_cuda_hook.c), recording every call's
 * inputs and output when a dump file is given. */
#include "pickle.h"
#include "pickle_fast.h"
#include "pickle_cuda.h"
#include <stdio.h>
#include <stdlib.h>

int  pickle_cuda_hook_attach(const pickle_fast_state_t* st, int device);
void pickle_cuda_hook_detach(void);
int  pickle_cuda_hook_call(const pickle_fast_state_t* st, int layer, size_t pos,
                           float* q, float* k, float* v, float* ao);

extern int (*pickle_fast_attn_hook)(const pickle_fast_state_t* state, int layer, size_t pos,
                                    float* q, float* k, float* v, float* ao);
extern FILE* e2e_dump_file;

static int dumping_hook(const pickle_fast_state_t* st, int layer, size_t pos,
                        float* q, float* k, float* v, float* ao) {
    size_t nq = (size_t)st->n_heads * st->head_dim, nk = (size_t)st->n_kv_heads * st->head_dim;
    int32_t hdr[2] = { layer, (int32_t)pos };
    fwrite(hdr, sizeof(int32_t), 2, e2e_dump_file);
    fwrite(q, sizeof(float), nq, e2e_dump_file);
    fwrite(k, sizeof(float), nk, e2e_dump_file);
    fwrite(v, sizeof(float), nk, e2e_dump_file);
    int rc = pickle_cuda_hook_call(st, layer, pos, q, k, v, ao);
    fwrite(ao, sizeof(float), nq, e2e_dump_file);
    return rc;
}

int e2e_attach(pickle_fast_state_t* st) {
    const char* dev = getenv("PICKLE_CUDA_DEVICE");
    int rc = pickle_cuda_hook_attach(st, dev ? atoi(dev) : 0);
    if (rc != PICKLE_OK) return rc;
    if (e2e_dump_file) pickle_fast_attn_hook = dumping_hook;
    return PICKLE_OK;
}

void e2e_detach(void) { pickle_cuda_hook_detach(); }
