// matvec_ex.h - library-internal forms of pickle_cuda_matvec_dev and
// pickle_cuda_matmul_dev (not exported). w_static: W is never written while
// it is in use (a loaded model's weights), so the tensor-core matvec may
// start streaming it before the previous kernel in the stream completes.
#pragma once
#include <cstddef>

int pcu_matvec_ex(int type, const void* W, int out_n, int in_n, int n_vec, const float* x, float* y, void* stream,
                  bool w_static);
int pcu_matmul_ex(int type, const void* W, int out_n, int in_n, int n_tok, const float* x, float* y,
                  void* workspace, size_t ws_bytes, void* stream, bool w_static);
