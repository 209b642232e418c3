// matvec_ex.h - library-internal forms of pickle_cuda_matvec_dev and
// pickle_cuda_matmul_dev (not exported). w_static: W is never written while
// it is in use (a loaded model's weights), so the tensor-core matvec may
// start streaming it before the previous kernel in the stream completes.
#pragma once
#include <cstddef>

int pcu_matvec_ex(int type, const void* W, int out_n, int in_n, int n_vec, const float* x, float* y, void* stream,
                  bool w_static);
// rowsc: the GEMM's per-row weight scales, precomputed by
// pcu_matmul_rowscale for constant weights (nullptr: computed per call).
int pcu_matmul_ex(int type, const void* W, int out_n, int in_n, int n_tok, const float* x, float* y,
                  void* workspace, size_t ws_bytes, void* stream, bool w_static, const float* rowsc);
// Those scales for W [out_n][in_n] of a quantized type (Q4_0, Q8_0, Q4_K, Q6_K).
int pcu_matmul_rowscale(int type, const void* W, int out_n, int in_n, float* rowsc, void* stream);
