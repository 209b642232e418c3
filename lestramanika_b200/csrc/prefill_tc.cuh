// prefill_tc.cuh - causal prefill on the tcgen05 tensor cores (BF16
// operands, F32 accumulation in TMEM).
#pragma once
#include "pcu_common.cuh"

inline bool prefill_tc_supported(int D, int G) { (void)D; (void)G; return false; }

inline int prefill_tc_launch(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, float* ao,
                             int n_seqs, int T, int H, int HK, int D, float scale, int* err, cudaStream_t st,
                             char* msg, size_t msg_len) {
    (void)q; (void)k; (void)v; (void)ao; (void)n_seqs; (void)T; (void)H; (void)HK; (void)D;
    (void)scale; (void)err; (void)st;
    snprintf(msg, msg_len, "tensor-core prefill not built");
    return -9;
}
