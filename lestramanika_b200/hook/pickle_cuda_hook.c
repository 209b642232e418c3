/*
 * pickle_cuda_hook.c - glue between pickle's forward pass and the B200 shim.
 *
 * Compiled together with a copy of lee-muriithi-kingori/lestramanika
 * src/pickle_fast.c patched by pickle_fast_cuda_hook.patch and built with
 * -DPICKLE_CUDA. The patch adds a function-pointer hook at the start of
 * the attention block (src/pickle_fast.c:1910); this file points it at
 * pickle_cuda_attn_decode, so each (token, layer) of pickle_fast_forward
 * runs RoPE + KV append + attention on the GPU, with the device KV cache
 * standing in for pickle_fast_kv_t (which stays allocated but unused).
 *
 * Usage, after pickle_fast_state_init (as pickle_chat_loop does at
 * src/pickle_host.c:433-440):
 *     pickle_cuda_hook_attach(&state, device);
 *     ... pickle_fast_forward(...) as before ...
 *     pickle_cuda_hook_detach();
 */
#include "pickle.h"
#include "pickle_fast.h"
#include "pickle_cuda.h"

extern int (*pickle_fast_attn_hook)(const pickle_fast_state_t* state, int layer, size_t pos,
                                    float* q, float* k, float* v, float* ao);

static pickle_cuda_t* g_cuda;
static const pickle_fast_state_t* g_state;

int pickle_cuda_hook_call(const pickle_fast_state_t* st, int layer, size_t pos,
                          float* q, float* k, float* v, float* ao) {
    if (!g_cuda || st != g_state) return PICKLE_ERR_ARG;
    return pickle_cuda_attn_decode(g_cuda, layer, pos, q, k, v, ao);
}

int pickle_cuda_hook_attach(const pickle_fast_state_t* st, int device) {
    if (!st) return PICKLE_ERR_ARG;
    if (g_cuda) { pickle_cuda_free(g_cuda); g_cuda = NULL; }
    pickle_cuda_params_t p;
    p.n_layers = st->n_layers;
    p.n_heads = st->n_heads;
    p.n_kv_heads = st->n_kv_heads;
    p.head_dim = st->head_dim;
    p.max_seq = st->max_seq;
    p.half = st->half;
    p.rope_inv_freq = st->rope_inv_freq;
    p.rope_theta = st->rope_theta;
    p.n_seqs = 1;
    p.rope_len = 0;
    int rc = pickle_cuda_init(&p, device, &g_cuda);
    if (rc != PICKLE_OK) { g_cuda = NULL; return rc; }
    g_state = st;
    pickle_fast_attn_hook = pickle_cuda_hook_call;
    return PICKLE_OK;
}

void pickle_cuda_hook_detach(void) {
    pickle_fast_attn_hook = 0;
    if (g_cuda) pickle_cuda_free(g_cuda);
    g_cuda = 0;
    g_state = 0;
}
