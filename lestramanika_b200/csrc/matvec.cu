// matvec.cu - y = W x on the GPU for pickle's weight formats, the
// projections either side of the attention block (q/k/v in, out after).
//
// Replaces pickle_fast_matmul_dispatch (lee-muriithi-kingori/lestramanika
// src/pickle_fast.c:1423-1474) for F32, F16, Q4_0, Q8_0, Q4_K and Q6_K
// weights, which are read in their raw on-disk block layout (the GGML
// formats: src/pickle_fast.c:161-196 Q4_0, :303-326 Q8_0, :563-738 Q4_K,
// :1084-1257 Q6_K, :1381-1419 F16). Like the reference's float paths, each
// weight is dequantized to float with the same per-element expression and
// multiplied by the float activation (no activation quantization), so the
// result matches within float rounding.
//
// Layout of the work: one warp takes kRows consecutive output rows; lane l
// handles elements 4l .. 4l+3 of every 128-element chunk of the row, so the
// weight bytes a warp instruction loads are one small contiguous range
// (coalesced even for 18- or 34-byte blocks, with naturally aligned 2- and
// 4-byte loads), and each float4 of x, read once, serves all kRows rows.
// n_vec activation vectors (1..8, e.g. a small decode batch) share one pass
// over the weights. Bound: HBM (the weight bytes).
#include "pickle_cuda.h"

#include <cuda_fp16.h>
#include <cstdint>

#include "matvec_tc.cuh"
#include "matmul_tc.cuh"
#include "matvec_ex.h"

namespace {

constexpr int kRows = 2;       // output rows per warp
constexpr int kWarps = 4;      // warps per CTA

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

__device__ __forceinline__ float ld_half(const unsigned char* p) {
    return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(p))));
}

// Four bytes at an even address.
__device__ __forceinline__ uint32_t ld4b_even(const unsigned char* p) {
    const unsigned short* q = reinterpret_cast<const unsigned short*>(p);
    return (uint32_t)__ldg(q) | ((uint32_t)__ldg(q + 1) << 16);
}

__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(signed char)((w >> (8 * i)) & 0xFF); }
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFF); }

// 6-bit scale and min of sub-block j (0..7) of a Q4_K block, from its 12
// packed bytes s: j < 4 in the low 6 bits of s[j] / s[j+4]; j >= 4 low 4
// bits from s[j+4], high 2 bits from the top of s[j-4] (scale) or s[j]
// (min) - the layout src/pickle_fast.c:368-383 decodes.
__device__ __forceinline__ void q4k_scale_min(const unsigned char* s, int j, int& sc, int& m) {
    if (j < 4) {
        sc = __ldg(s + j) & 63;
        m = __ldg(s + j + 4) & 63;
    } else {
        const int a = __ldg(s + j + 4);
        sc = (a & 15) | ((__ldg(s + j - 4) >> 6) << 4);
        m = (a >> 4) | ((__ldg(s + j) >> 6) << 4);
    }
}

// Dequantized weights of elements e .. e+3 (e % 4 == 0) of one row.
template <int TYPE>
__device__ __forceinline__ float4 dq4(const unsigned char* row, int e);

template <>
__device__ __forceinline__ float4 dq4<T_F32>(const unsigned char* row, int e) {
    return __ldg(reinterpret_cast<const float4*>(row) + e / 4);
}

template <>
__device__ __forceinline__ float4 dq4<T_F16>(const unsigned char* row, int e) {
    const uint2 h = __ldg(reinterpret_cast<const uint2*>(row) + e / 4);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// Q4_0: 18 bytes / 32 elements: d (f16), then byte i holds element i (low
// nibble) and element 16 + i (high nibble), both offset by -8.
template <>
__device__ __forceinline__ float4 dq4<T_Q4_0>(const unsigned char* row, int e) {
    const unsigned char* blk = row + (size_t)(e / 32) * 18;
    const float d = ld_half(blk);
    const int w = e % 32;
    const uint32_t b = ld4b_even(blk + 2 + (w & 15));
    const int sh = w < 16 ? 0 : 4;
    return make_float4(d * (float)(((ubyte(b, 0) >> sh) & 15) - 8), d * (float)(((ubyte(b, 1) >> sh) & 15) - 8),
                       d * (float)(((ubyte(b, 2) >> sh) & 15) - 8), d * (float)(((ubyte(b, 3) >> sh) & 15) - 8));
}

// Q8_0: 34 bytes / 32 elements: d (f16), then 32 signed bytes.
template <>
__device__ __forceinline__ float4 dq4<T_Q8_0>(const unsigned char* row, int e) {
    const unsigned char* blk = row + (size_t)(e / 32) * 34;
    const float d = ld_half(blk);
    const uint32_t b = ld4b_even(blk + 2 + e % 32);
    return make_float4(d * (float)sbyte(b, 0), d * (float)sbyte(b, 1), d * (float)sbyte(b, 2), d * (float)sbyte(b, 3));
}

// Q4_K: 144 bytes / 256 elements: d, dmin (f16), 12 bytes of 6-bit
// sub-block scales and mins, then 128 bytes of 4-bit quants. Chunk c (64
// elements) uses qs[32c .. 32c+31]: element 64c + l is the low nibble of
// qs[32c + l] with sub-block 2c, element 64c + 32 + l the high nibble with
// sub-block 2c + 1; weight = d * scale * q - dmin * min.
template <>
__device__ __forceinline__ float4 dq4<T_Q4_K>(const unsigned char* row, int e) {
    const unsigned char* blk = row + (size_t)(e / 256) * 144;
    const int w = e % 256, c = w / 64, r = w % 64, hi = r >= 32, l = r & 31;
    int sc, m;
    q4k_scale_min(blk + 4, 2 * c + hi, sc, m);
    const float d1 = ld_half(blk) * (float)sc, m1 = ld_half(blk + 2) * (float)m;
    const uint32_t b = __ldg(reinterpret_cast<const uint32_t*>(blk + 16 + 32 * c + l));
    const int sh = hi ? 4 : 0;
    return make_float4(d1 * (float)((ubyte(b, 0) >> sh) & 15) - m1, d1 * (float)((ubyte(b, 1) >> sh) & 15) - m1,
                       d1 * (float)((ubyte(b, 2) >> sh) & 15) - m1, d1 * (float)((ubyte(b, 3) >> sh) & 15) - m1);
}

// Q6_K: 210 bytes / 256 elements: ql[128] (low 4 bits), qh[64] (high 2
// bits), 16 signed 8-bit scales, d (f16). Half n (128 elements) uses
// ql[64n ..], qh[32n ..], scales[8n ..]; for l < 32 and quarter t (0..3),
// element 128n + 32t + l has low bits from ql[64n + l + 32 (t & 1)] (low
// nibble for t < 2, high for t >= 2), high bits (qh[32n + l] >> 2t) & 3,
// value q - 32 and scale scales[8n + l / 16 + 2t]; weight = d * scale * q.
template <>
__device__ __forceinline__ float4 dq4<T_Q6_K>(const unsigned char* row, int e) {
    const unsigned char* blk = row + (size_t)(e / 256) * 210;
    const int w = e % 256, n = w / 128, r = w % 128, t = r / 32, l = r & 31;
    const float ds = ld_half(blk + 208) * (float)(signed char)__ldg(blk + 192 + 8 * n + l / 16 + 2 * t);
    const uint32_t lo = ld4b_even(blk + 64 * n + l + 32 * (t & 1));
    const uint32_t hb = ld4b_even(blk + 128 + 32 * n + l);
    const int sl = t >= 2 ? 4 : 0, sh = 2 * t;
    float v[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i)
        v[i] = ds * (float)((((ubyte(lo, i) >> sl) & 15) | (((ubyte(hb, i) >> sh) & 3) << 4)) - 32);
    return make_float4(v[0], v[1], v[2], v[3]);
}

template <int TYPE, int NV>
__global__ void __launch_bounds__(kWarps * 32) matvec_kernel(const unsigned char* __restrict__ W, size_t row_bytes,
                                                             int out_n, int in_n, const float* __restrict__ x,
                                                             float* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (blockIdx.x * kWarps + warp) * kRows;
    if (r0 >= out_n) return;
    const int nr = out_n - r0 < kRows ? out_n - r0 : kRows;
    float acc[kRows][NV];
    #pragma unroll
    for (int r = 0; r < kRows; ++r)
        #pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = 0.f;
    #pragma unroll 2
    for (int e = 4 * lane; e < in_n; e += 128) {
        float4 xv[NV];
        #pragma unroll
        for (int v = 0; v < NV; ++v) xv[v] = __ldg(reinterpret_cast<const float4*>(x + (size_t)v * in_n + e));
        #pragma unroll
        for (int r = 0; r < kRows; ++r) {
            if (r < nr) {
                const float4 w = dq4<TYPE>(W + (size_t)(r0 + r) * row_bytes, e);
                #pragma unroll
                for (int v = 0; v < NV; ++v) {
                    float a = acc[r][v];
                    a = fmaf(w.x, xv[v].x, a);
                    a = fmaf(w.y, xv[v].y, a);
                    a = fmaf(w.z, xv[v].z, a);
                    a = fmaf(w.w, xv[v].w, a);
                    acc[r][v] = a;
                }
            }
        }
    }
    #pragma unroll
    for (int r = 0; r < kRows; ++r)
        #pragma unroll
        for (int v = 0; v < NV; ++v) {
            float a = acc[r][v];
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0 && r < nr) y[(size_t)v * out_n + r0 + r] = a;
        }
}

template <int TYPE>
cudaError_t launch_type(const unsigned char* W, size_t row_bytes, int out_n, int in_n, int n_vec, const float* x,
                        float* y, cudaStream_t st) {
    const unsigned grid = (unsigned)((out_n + kRows * kWarps - 1) / (kRows * kWarps));
    switch (n_vec) {
#define PCU_MV(N) case N: matvec_kernel<TYPE, N><<<grid, kWarps * 32, 0, st>>>(W, row_bytes, out_n, in_n, x, y); break;
        PCU_MV(1) PCU_MV(2) PCU_MV(3) PCU_MV(4) PCU_MV(5) PCU_MV(6) PCU_MV(7) PCU_MV(8)
#undef PCU_MV
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace

// pickle_cuda_matvec_dev, and for the model's own projections (w_static:
// W is never written while the model lives) the same with the weight
// stream of the tensor-core kernel started before the previous kernel in
// the stream has finished.
int pcu_matvec_ex(int type, const void* W, int out_n, int in_n, int n_vec, const float* x, float* y, void* stream,
                  bool w_static) {
    if (!W || !x || !y || out_n < 1 || in_n < 1 || n_vec < 1 || n_vec > PICKLE_CUDA_MATVEC_MAX_VEC)
        return PICKLE_ERR_ARG;
    if (((uintptr_t)W | (uintptr_t)x | (uintptr_t)y) % 16) return PICKLE_ERR_ARG;
    size_t row_bytes = 0;
    int qk = 4;
    switch (type) {
        case T_F32: row_bytes = (size_t)in_n * 4; qk = 4; break;
        case T_F16: row_bytes = (size_t)in_n * 2; qk = 4; break;
        case T_Q4_0: row_bytes = (size_t)(in_n / 32) * 18; qk = 32; break;
        case T_Q8_0: row_bytes = (size_t)(in_n / 32) * 34; qk = 32; break;
        case T_Q4_K: row_bytes = (size_t)(in_n / 256) * 144; qk = 256; break;
        case T_Q6_K: row_bytes = (size_t)(in_n / 256) * 210; qk = 256; break;
        default: return PICKLE_ERR_TYPE;
    }
    if (in_n % qk) return PICKLE_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned char* w = static_cast<const unsigned char*>(W);
    cudaError_t e = cudaErrorInvalidValue;
    switch (type) {
        case T_F32: e = launch_type<T_F32>(w, row_bytes, out_n, in_n, n_vec, x, y, st); break;
        case T_F16:
            e = mvtc::tc_supported<T_F16>(w, row_bytes, in_n)
                    ? mvtc::launch<T_F16>(w, row_bytes, out_n, in_n, n_vec, x, y, st, w_static)
                    : launch_type<T_F16>(w, row_bytes, out_n, in_n, n_vec, x, y, st);
            break;
        case T_Q4_0:
            e = mvtc::tc_supported<T_Q4_0>(w, row_bytes, in_n)
                    ? mvtc::launch<T_Q4_0>(w, row_bytes, out_n, in_n, n_vec, x, y, st, w_static)
                    : launch_type<T_Q4_0>(w, row_bytes, out_n, in_n, n_vec, x, y, st);
            break;
        case T_Q8_0:
            e = mvtc::tc_supported<T_Q8_0>(w, row_bytes, in_n)
                    ? mvtc::launch<T_Q8_0>(w, row_bytes, out_n, in_n, n_vec, x, y, st, w_static)
                    : launch_type<T_Q8_0>(w, row_bytes, out_n, in_n, n_vec, x, y, st);
            break;
        case T_Q4_K:
            e = mvtc::tc_supported<T_Q4_K>(w, row_bytes, in_n)
                    ? mvtc::launch<T_Q4_K>(w, row_bytes, out_n, in_n, n_vec, x, y, st, w_static)
                    : launch_type<T_Q4_K>(w, row_bytes, out_n, in_n, n_vec, x, y, st);
            break;
        case T_Q6_K:
            e = mvtc::tc_supported<T_Q6_K>(w, row_bytes, in_n)
                    ? mvtc::launch<T_Q6_K>(w, row_bytes, out_n, in_n, n_vec, x, y, st, w_static)
                    : launch_type<T_Q6_K>(w, row_bytes, out_n, in_n, n_vec, x, y, st);
            break;
    }
    return e == cudaSuccess ? PICKLE_OK : PICKLE_ERR_DEVICE;
}

extern "C" PICKLE_CUDA_API int pickle_cuda_matvec_dev(int type, const void* W, int out_n, int in_n, int n_vec,
                                                      const float* x, float* y, void* stream) {
    return pcu_matvec_ex(type, W, out_n, in_n, n_vec, x, y, stream, false);
}

extern "C" PICKLE_CUDA_API size_t pickle_cuda_matvec_row_bytes(int type, int in_n) {
    switch (type) {
        case T_F32: return (size_t)in_n * 4;
        case T_F16: return (size_t)in_n * 2;
        case T_Q4_0: return in_n % 32 ? 0 : (size_t)(in_n / 32) * 18;
        case T_Q8_0: return in_n % 32 ? 0 : (size_t)(in_n / 32) * 34;
        case T_Q4_K: return in_n % 256 ? 0 : (size_t)(in_n / 256) * 144;
        case T_Q6_K: return in_n % 256 ? 0 : (size_t)(in_n / 256) * 210;
        default: return 0;
    }
}

extern "C" PICKLE_CUDA_API int pickle_cuda_matvec_take_error(int device, int* code) {
    if (!code) return PICKLE_ERR_ARG;
    if (cudaSetDevice(device) != cudaSuccess) return PICKLE_ERR_DEVICE;
    int v = 0;
    const int zero = 0;
    if (cudaMemcpyFromSymbol(&v, mvtc::g_mv_err, sizeof(int)) != cudaSuccess ||
        cudaMemcpyToSymbol(mvtc::g_mv_err, &zero, sizeof(int)) != cudaSuccess)
        return PICKLE_ERR_DEVICE;
    *code = v;
    return PICKLE_OK;
}

extern "C" PICKLE_CUDA_API size_t pickle_cuda_matmul_workspace(int out_n, int in_n, int n_tok) {
    if (out_n < 1 || in_n < 1 || n_tok < 1) return 0;
    return mmtc::workspace_bytes(out_n, in_n, n_tok);
}

int pcu_matmul_ex(int type, const void* W, int out_n, int in_n, int n_tok, const float* x, float* y,
                  void* workspace, size_t ws_bytes, void* stream, bool w_static, const float* rowsc) {
    if (!W || !x || !y || out_n < 1 || in_n < 1 || n_tok < 1) return PICKLE_ERR_ARG;
    if (((uintptr_t)W | (uintptr_t)x | (uintptr_t)y) % 16) return PICKLE_ERR_ARG;
    if (type != T_F32 && type != T_F16 && type != T_Q4_0 && type != T_Q8_0 && type != T_Q4_K && type != T_Q6_K)
        return PICKLE_ERR_TYPE;
    const size_t row_bytes = pickle_cuda_matvec_row_bytes(type, in_n);
    if (row_bytes == 0) return PICKLE_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned char* w = static_cast<const unsigned char*>(W);
    const bool ws_ok = workspace && (uintptr_t)workspace % 256 == 0 &&
                       ws_bytes >= mmtc::workspace_bytes(out_n, in_n, n_tok);
    // A few rows of a model's constant weights (a decode batch) stay on the
    // matvec unless it would need more than three passes over W, because
    // not enough of the rows fit in its shared memory at once.
    int fit = PICKLE_CUDA_MATVEC_MAX_VEC;
    if (w_static && n_tok > 1) {
        switch (type) {
            case T_F16: fit = mvtc::fit_nv<T_F16>(in_n); break;
            case T_Q4_0: fit = mvtc::fit_nv<T_Q4_0>(in_n); break;
            case T_Q8_0: fit = mvtc::fit_nv<T_Q8_0>(in_n); break;
            case T_Q4_K: fit = mvtc::fit_nv<T_Q4_K>(in_n); break;
            case T_Q6_K: fit = mvtc::fit_nv<T_Q6_K>(in_n); break;
        }
    }
    const bool gemm = n_tok > PICKLE_CUDA_MATVEC_MAX_VEC || (w_static && (n_tok + fit - 1) / fit > 3);
    if (gemm && ws_ok && type != T_F32 && mmtc::supported(w, row_bytes, in_n)) {
        cudaError_t e = cudaErrorInvalidValue;
        switch (type) {
            case T_F16: e = mmtc::launch<T_F16>(w, row_bytes, out_n, in_n, n_tok, x, y, workspace, st, rowsc); break;
            case T_Q4_0: e = mmtc::launch<T_Q4_0>(w, row_bytes, out_n, in_n, n_tok, x, y, workspace, st, rowsc); break;
            case T_Q8_0: e = mmtc::launch<T_Q8_0>(w, row_bytes, out_n, in_n, n_tok, x, y, workspace, st, rowsc); break;
            case T_Q4_K: e = mmtc::launch<T_Q4_K>(w, row_bytes, out_n, in_n, n_tok, x, y, workspace, st, rowsc); break;
            case T_Q6_K: e = mmtc::launch<T_Q6_K>(w, row_bytes, out_n, in_n, n_tok, x, y, workspace, st, rowsc); break;
        }
        return e == cudaSuccess ? PICKLE_OK : PICKLE_ERR_DEVICE;
    }
    // Otherwise: the matvec, up to eight activation rows per pass over W.
    for (int v0 = 0; v0 < n_tok; v0 += PICKLE_CUDA_MATVEC_MAX_VEC) {
        const int nv = n_tok - v0 < PICKLE_CUDA_MATVEC_MAX_VEC ? n_tok - v0 : PICKLE_CUDA_MATVEC_MAX_VEC;
        const int rc = pcu_matvec_ex(type, W, out_n, in_n, nv, x + (size_t)v0 * in_n, y + (size_t)v0 * out_n,
                                     stream, w_static);
        if (rc != PICKLE_OK) return rc;
    }
    return PICKLE_OK;
}

extern "C" PICKLE_CUDA_API int pickle_cuda_matmul_dev(int type, const void* W, int out_n, int in_n, int n_tok,
                                                      const float* x, float* y, void* workspace, size_t ws_bytes,
                                                      void* stream) {
    return pcu_matmul_ex(type, W, out_n, in_n, n_tok, x, y, workspace, ws_bytes, stream, false, nullptr);
}

int pcu_matmul_rowscale(int type, const void* W, int out_n, int in_n, float* rowsc, void* stream) {
    const size_t row_bytes = pickle_cuda_matvec_row_bytes(type, in_n);
    if (!W || !rowsc || out_n < 1 || row_bytes == 0) return PICKLE_ERR_ARG;
    const uint8_t* w = static_cast<const uint8_t*>(W);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    switch (type) {
        case T_Q4_0: e = mmtc::rowscale<T_Q4_0>(w, row_bytes, out_n, in_n, rowsc, st); break;
        case T_Q8_0: e = mmtc::rowscale<T_Q8_0>(w, row_bytes, out_n, in_n, rowsc, st); break;
        case T_Q4_K: e = mmtc::rowscale<T_Q4_K>(w, row_bytes, out_n, in_n, rowsc, st); break;
        case T_Q6_K: e = mmtc::rowscale<T_Q6_K>(w, row_bytes, out_n, in_n, rowsc, st); break;
        default: return PICKLE_ERR_TYPE;
    }
    return e == cudaSuccess ? PICKLE_OK : PICKLE_ERR_DEVICE;
}
