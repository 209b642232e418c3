/* TEST INFRASTRUCTURE ONLY: adapter that serves the hook-patched forward
 * pass's attention block with the CPU oracle (ref_attn_cpu.c). Used to
 * certify that the oracle reproduces the reference's logits bit for bit. */
#include "pickle.h"
#include "pickle_fast.h"
#include <stdio.h>
#include <string.h>
#include <stdlib.h>

typedef struct oracle_attn oracle_attn_t;
int  oracle_attn_create(int n_layers, int n_heads, int n_kv_heads, int head_dim,
                        int max_seq, float theta, oracle_attn_t** out);
void oracle_attn_destroy(oracle_attn_t* o);
int  oracle_attn_decode(oracle_attn_t* o, int layer, size_t pos,
                        float* q, float* k, const float* v, float* ao);

extern int (*pickle_fast_attn_hook)(const pickle_fast_state_t* state, int layer, size_t pos,
                                    float* q, float* k, float* v, float* ao);
extern FILE* e2e_dump_file;

static oracle_attn_t* g_oracle;

static int oracle_hook(const pickle_fast_state_t* st, int layer, size_t pos,
                       float* q, float* k, float* v, float* ao) {
    size_t nq = (size_t)st->n_heads * st->head_dim, nk = (size_t)st->n_kv_heads * st->head_dim;
    if (e2e_dump_file) {
        int32_t hdr[2] = { layer, (int32_t)pos };
        fwrite(hdr, sizeof(int32_t), 2, e2e_dump_file);
        fwrite(q, sizeof(float), nq, e2e_dump_file);
        fwrite(k, sizeof(float), nk, e2e_dump_file);
        fwrite(v, sizeof(float), nk, e2e_dump_file);
    }
    int rc = oracle_attn_decode(g_oracle, layer, pos, q, k, v, ao);
    if (e2e_dump_file) fwrite(ao, sizeof(float), nq, e2e_dump_file);
    return rc;
}

int e2e_attach(pickle_fast_state_t* st) {
    int rc = oracle_attn_create(st->n_layers, st->n_heads, st->n_kv_heads, st->head_dim,
                                st->max_seq, st->rope_theta, &g_oracle);
    if (rc != 0) return rc;
    pickle_fast_attn_hook = oracle_hook;
    return PICKLE_OK;
}

void e2e_detach(void) {
    pickle_fast_attn_hook = NULL;
    oracle_attn_destroy(g_oracle);
    g_oracle = NULL;
}
