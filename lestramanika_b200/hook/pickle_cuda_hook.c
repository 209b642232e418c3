/*
 * pickle_cuda_hook.c - glue between pickle's forward pass and the B200 shim.
 *
 * Compiled together with a copy of lee-muriithi-kingori/lestramanika
 * src/pickle_fast.c patched by pickle_fast_cuda_hook.patch and built with
 * -DPICKLE_CUDA (the PICKLE_CUDA=1 target of pickle_makefile_cuda.patch).
 * The patch delegates the attention block (src/pickle_fast.c:1910-2109:
 * RoPE, KV append, causal attention) to this file, so each (token, layer)
 * of pickle_fast_forward runs on the GPU through pickle_cuda_attn_decode,
 * with the device KV cache standing in for pickle_fast_kv_t (which stays
 * allocated but unused).
 *
 * Two ways in:
 *   - automatic: the unmodified callers (pickle_chat_loop,
 *     src/pickle_host.c:410-535, and so `./pickle infer` / `chat` / `bench`)
 *     need no change. The first attention call of a state creates the
 *     device handle from that state's dimensions (pickle_fast_state_t,
 *     src/pickle_fast.h:55-123) on device $PICKLE_CUDA_DEVICE (default 0);
 *     a state with other dimensions replaces it. Positions index the
 *     device cache exactly as kv_pos indexes the host one, so a new
 *     conversation simply overwrites rows from position 0.
 *   - explicit, after pickle_fast_state_init:
 *         pickle_cuda_hook_attach(&state, device);
 *         ... pickle_fast_forward(...) as before ...
 *         pickle_cuda_hook_detach();
 * A failure (no GPU, a CUDA error) is returned to pickle_fast_forward as
 * the shim's PICKLE_ERR_* code; there is no silent CPU fallback. With
 * PICKLE_CUDA_VERBOSE set, the device set-up is reported on stderr.
 * Like pickle_fast_forward itself, this is not re-entrant: one host thread
 * drives one state.
 */
#include "pickle.h"
#include "pickle_fast.h"
#include "pickle_cuda.h"

#include <stdio.h>
#include <stdlib.h>

extern int (*pickle_fast_attn_hook)(const pickle_fast_state_t* state, int layer, size_t pos,
                                    float* q, float* k, float* v, float* ao);

static pickle_cuda_t* g_cuda;
static const pickle_fast_state_t* g_state;
static int g_dims[7];          /* n_layers, H, HK, D, max_seq, half, device of g_cuda */

static void state_dims(const pickle_fast_state_t* st, int device, int* d) {
    d[0] = st->n_layers; d[1] = st->n_heads; d[2] = st->n_kv_heads; d[3] = st->head_dim;
    d[4] = st->max_seq; d[5] = st->half; d[6] = device;
}

static int open_device(const pickle_fast_state_t* st, int device) {
    if (g_cuda) { pickle_cuda_free(g_cuda); g_cuda = NULL; g_state = NULL; }
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
    if (rc != PICKLE_OK) {
        g_cuda = NULL;
        fprintf(stderr, "pickle_cuda: device %d set-up failed (rc=%d)\n", device, rc);
        return rc;
    }
    g_state = st;
    state_dims(st, device, g_dims);
    if (getenv("PICKLE_CUDA_VERBOSE"))
        fprintf(stderr, "pickle_cuda: attention of %d layers (%d q / %d kv heads, head_dim %d) on device %d\n",
                st->n_layers, st->n_heads, st->n_kv_heads, st->head_dim, device);
    return PICKLE_OK;
}

int pickle_cuda_hook_call(const pickle_fast_state_t* st, int layer, size_t pos,
                          float* q, float* k, float* v, float* ao) {
    if (!g_cuda || st != g_state) return PICKLE_ERR_ARG;
    return pickle_cuda_attn_decode(g_cuda, layer, pos, q, k, v, ao);
}

int pickle_cuda_hook_auto(const pickle_fast_state_t* st, int layer, size_t pos,
                          float* q, float* k, float* v, float* ao) {
    if (!st) return PICKLE_ERR_ARG;
    const char* dv = getenv("PICKLE_CUDA_DEVICE");
    const int device = dv ? atoi(dv) : 0;
    int d[7];
    state_dims(st, device, d);
    int same = g_cuda != NULL;
    for (int i = 0; i < 7 && same; ++i) same = d[i] == g_dims[i];
    if (!same) {
        int rc = open_device(st, device);
        if (rc != PICKLE_OK) return rc;
    }
    g_state = st;
    return pickle_cuda_attn_decode(g_cuda, layer, pos, q, k, v, ao);
}

int pickle_cuda_hook_attach(const pickle_fast_state_t* st, int device) {
    if (!st) return PICKLE_ERR_ARG;
    int rc = open_device(st, device);
    if (rc != PICKLE_OK) return rc;
    pickle_fast_attn_hook = pickle_cuda_hook_call;
    return PICKLE_OK;
}

void pickle_cuda_hook_detach(void) {
    pickle_fast_attn_hook = 0;
    if (g_cuda) pickle_cuda_free(g_cuda);
    g_cuda = 0;
    g_state = 0;
}
