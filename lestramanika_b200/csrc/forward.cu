// forward.cu - pickle_fast_forward on the device.
//
// The reference's forward pass (lee-muriithi-kingori/lestramanika
// src/pickle_fast.c:1822-2184) runs every prompt token through every layer on
// the host:
//   x = token_embd[tok]                                        :1887-1897
//   per layer L:
//     xn = rmsnorm(x, attn_norm)                               :1899-1901
//     q, k, v = Wq xn, Wk xn, Wv xn                            :1903-1908
//     ao = attention block (RoPE, cache append, softmax . V)   :1910-2109
//     x += Wo ao                                               :2112-2114
//     xn2 = rmsnorm(x, ffn_norm)                               :2117-2118
//     act = silu(Wgate xn2) * (Wup xn2)                        :2120-2131
//     x += Wdown act                                           :2133-2135
//   last token: x = rmsnorm(x, output_norm); logits = Wout x   :2138-2174
// and the caller picks the next token with pickle_fast_argmax (:2186-2194).
//
// Here all of it stays in HBM: the weights are uploaded once, in their raw
// GGML blocks, into one allocation; a prompt chunk of T tokens goes through
// each projection as one GEMM (pickle_cuda_matmul_dev) and through the
// attention block as one causal prefill (pickle_cuda_prefill_dev); a decode
// step (T = 1) uses the matvec and the split-KV decode. The elementwise work
// of the reference's loop is fused into small kernels below (norm with the
// residual add before it, embedding with the first norm, SwiGLU, argmax,
// the temperature / top-p sampler). The decode loop feeds each chosen id
// back on the device, so a generation of n tokens needs no host round trip
// per token. With n_seqs cache slots, one step can also decode many
// sequences together, each at its own position (continuous batching).
#include "pickle_cuda.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "matvec_ex.h"
#include "pcu_common.cuh"

namespace {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

constexpr int kNormThreads = 512;
constexpr int kArgmaxThreads = 1024;
constexpr int kLayerTensors = PICKLE_CUDA_LAYER_TENSORS;
constexpr int kMaxNormVec = 16;      // float4s per thread: rows up to 4 * 16 * 512 = 32768 floats

// Block-wide float sum (kNormThreads threads); every thread gets the total.
__device__ float block_sum(float v) {
    __shared__ float part[kNormThreads / 32];
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) part[w] = v;
    __syncthreads();
    float t = l < kNormThreads / 32 ? part[l] : 0.0f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

__device__ __forceinline__ float sumsq4(float4 a) { return a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w; }

// pickle_fast_rmsnorm (src/pickle_fast.c:114-120) of the row held in v
// (thread-strided float4s) into xn:
//   rsq = 1 / sqrtf(sum(x^2) / n + eps);  xn[i] = x[i] * w[i] * rsq.
// w == nullptr copies x (a model without output_norm, state->t_norm < 0).
template <int V>
__device__ void norm_row(const float4 (&v)[V], const float* w, float* xn, int n, float eps, float ss) {
    const int n4 = n >> 2;
    float4* o = reinterpret_cast<float4*>(xn);
    const float rsq = w ? 1.0f / sqrtf(ss / (float)n + eps) : 1.0f;
    const float4* w4 = reinterpret_cast<const float4*>(w);
    #pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < n4) {
            if (!w) {
                o[i] = v[j];
            } else {
                const float4 ww = w4[i];
                o[i] = make_float4((v[j].x * ww.x) * rsq, (v[j].y * ww.y) * rsq, (v[j].z * ww.z) * rsq,
                                   (v[j].w * ww.w) * rsq);
            }
        }
    }
}

// One CTA per token row r = blockIdx.x: x[r] += delta[r] (the residual add
// after a projection, skipped when delta is null), then
// xn[r] = rmsnorm(x[r], w). n is a multiple of 4 and at most
// 4 * V * kNormThreads; each thread keeps its V float4s in registers.
// Launched with programmatic stream serialization.
template <int V>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                                   const float* __restrict__ w, float* __restrict__ xn,
                                                                   int n, float eps) {
    griddep_launch_dependents();
    griddep_wait();
    const size_t r = blockIdx.x;
    const int n4 = n >> 2;
    float4* xr = reinterpret_cast<float4*>(x + r * n);
    const float4* dr = delta ? reinterpret_cast<const float4*>(delta + r * n) : nullptr;
    float4 v[V];
    float ss = 0.0f;
    #pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n4) {
            float4 a = xr[i];
            if (dr) {
                const float4 d = dr[i];
                a = make_float4(a.x + d.x, a.y + d.y, a.z + d.z, a.w + d.w);
                xr[i] = a;
            }
            v[j] = a;
            ss += sumsq4(a);
        }
    }
    ss = block_sum(ss);
    norm_row<V>(v, w, xn + r * n, n, eps, ss);
}

// Embedding lookup (src/pickle_fast.c:1887-1897: F32 rows, or F16 rows
// converted exactly) fused with the first layer's attention norm. A token
// outside [0, vocab) is recorded as PCU_DEVERR_ARG and looked up as 0; the
// host entry points check host tokens before they are uploaded.
template <int V>
__global__ void __launch_bounds__(kNormThreads) embed_rmsnorm_kernel(const int32_t* __restrict__ tok,
                                                                     const void* __restrict__ emb, int emb_f16,
                                                                     int vocab, const float* __restrict__ w,
                                                                     float* __restrict__ x, float* __restrict__ xn,
                                                                     int n, float eps, int* err) {
    griddep_launch_dependents();
    griddep_wait();
    const size_t r = blockIdx.x;
    int t = tok[r];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0) record_error(err, PCU_DEVERR_ARG);
        t = 0;
    }
    const int n4 = n >> 2;
    float4* xr = reinterpret_cast<float4*>(x + r * n);
    float4 v[V];
    float ss = 0.0f;
    #pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n4) {
            float4 a;
            if (emb_f16) {
                const uint2 h = reinterpret_cast<const uint2*>(static_cast<const __half*>(emb) + (size_t)t * n)[i];
                const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                a = make_float4(lo.x, lo.y, hi.x, hi.y);
            } else {
                a = reinterpret_cast<const float4*>(static_cast<const float*>(emb) + (size_t)t * n)[i];
            }
            xr[i] = a;
            v[j] = a;
            ss += sumsq4(a);
        }
    }
    ss = block_sum(ss);
    norm_row<V>(v, w, xn + r * n, n, eps, ss);
}

// SwiGLU (src/pickle_fast.c:2124-2131) over T rows of ID:
//   act[t][i] = g * (1 / (1 + expf(-g))) * up,  g = gate[t * ld + i],
//   up = gate[t * ld + up_off + i]
// (gate and up either one [T][2 ID] output of the fused projection, or
// act == gate with up_off the distance to a separate up buffer and ld = ID).
__global__ void swiglu_kernel(const float* __restrict__ gate, long long up_off, long long ld, int ID, int T,
                              float* act) {
    griddep_launch_dependents();
    griddep_wait();
    const size_t n = (size_t)T * ID;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
        const size_t t = e / ID, i = e - t * ID;
        const float gv = gate[t * ld + i];
        const float up = gate[t * ld + up_off + i];
        const float sig = 1.0f / (1.0f + expf(-gv));
        act[e] = gv * sig * up;
    }
}

// ---- Sampling: pickle_fast_sample_temp (src/pickle_fast.c:2204-2276) ----
// One CTA of kSampleThreads. The reference, for temp > 0:
//   logits /= temp; e = expf(logits - max); sum = sum(e);  (0 if sum == 0)
//   r = (xorshift32(seed) & 0xFFFFFF) / (float)0xFFFFFF
//   0 < top_p < 1: the fewest largest p = e / sum whose running sum cum
//     reaches top_p (a selection sort), then the first of them, largest
//     first, at which the running sum reaches r * cum (else the largest);
//   otherwise the first index at which the running sum of p reaches r
//     (else n - 1).
// Here the sums are fixed-order trees instead of one running float sum, so
// a draw within float rounding of a boundary may pick the neighbour; the
// nucleus is found without sorting, by binary searches over the bit
// patterns of e (non-negative floats order like their bits); among equal
// values the lower index comes first. logits are left holding e, as the
// reference leaves them.
constexpr int kSampleThreads = 1024;

template <int NT>
__device__ float block_sum_n(float v, float* part) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) part[w] = v;
    __syncthreads();
    float t = l < NT / 32 ? part[l] : 0.0f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

template <int NT>
__device__ float block_max_n(float v, float* part) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) part[w] = v;
    __syncthreads();
    float t = l < NT / 32 ? part[l] : -INFINITY;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    return t;
}

template <int NT>
__device__ int block_min_i(int v, int* part) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) part[w] = v;
    __syncthreads();
    int t = l < NT / 32 ? part[l] : INT32_MAX;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = min(t, __shfl_xor_sync(0xffffffffu, t, o));
    return t;
}

// Exclusive scan in thread order (one value per thread); every thread gets its prefix.
template <int NT, typename T>
__device__ T block_excl_scan(T v, T* part) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    T inc = v;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T t = __shfl_up_sync(0xffffffffu, inc, o);
        if (l >= o) inc += t;
    }
    __syncthreads();
    if (l == 31) part[w] = inc;
    __syncthreads();
    T base = 0;
    for (int j = 0; j < w; ++j) base += part[j];
    return base + inc - v;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(float* __restrict__ lg, int n, float temp,
                                                                float top_p, uint32_t seed, int32_t* __restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr int NT = kSampleThreads;
    __shared__ float fpart[NT / 32];
    __shared__ int ipart[NT / 32];
    const int tid = threadIdx.x;
    float mx = -INFINITY;
    for (int i = tid; i < n; i += NT) {
        const float l = lg[i] / temp;
        lg[i] = l;
        mx = fmaxf(mx, l);
    }
    mx = block_max_n<NT>(mx, fpart);
    float s = 0.0f;
    for (int i = tid; i < n; i += NT) {
        const float e = expf(lg[i] - mx);
        lg[i] = e;
        s += e;
    }
    const float sum = block_sum_n<NT>(s, fpart);
    uint32_t x = seed ? seed : 0x12345678u;   // g_rng_state, then one xorshift32 step
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    const float r = (float)(x & 0xFFFFFFu) / (float)0xFFFFFF;
    if (sum == 0.0f) {
        if (tid == 0) *out = 0;
        return;
    }
    // Each thread's contiguous run of indices, for the scans in index order.
    const int C = (n + NT - 1) / NT;
    const int i0 = min(n, tid * C), i1 = min(n, i0 + C);
    if (top_p > 0.0f && top_p < 1.0f) {
        // sum of p over the elements whose e has bits >= b
        auto sum_ge = [&](uint32_t b) {
            float a = 0.0f;
            for (int i = tid; i < n; i += NT) {
                const float e = lg[i];
                if (__float_as_uint(e) >= b) a += e / sum;
            }
            return block_sum_n<NT>(a, fpart);
        };
        auto count_eq = [&](uint32_t b) {
            float c = 0.0f;
            for (int i = tid; i < n; i += NT) c += __float_as_uint(lg[i]) == b ? 1.0f : 0.0f;
            return (int)block_sum_n<NT>(c, fpart);
        };
        // Largest bits b with sum_ge(b) >= v (lo0 when none qualifies); at most 31 steps.
        auto search = [&](uint32_t lo0, float v) {
            uint32_t lo = lo0, hi = 0x3F800001u;            // e <= 1 = expf(0)
            while (hi - lo > 1) {
                const uint32_t mid = lo + (hi - lo) / 2;
                if (sum_ge(mid) >= v) lo = mid; else hi = mid;
            }
            return lo;
        };
        // The nucleus: every e above bk, then equal ones until cum >= top_p.
        const uint32_t bk = search(0u, top_p);
        const float pk = __uint_as_float(bk) / sum;
        float cum = sum_ge(bk + 1);
        const int eq_k = count_eq(bk);
        int take_k = 0;
        while (take_k < eq_k && cum < top_p) {
            cum += pk;
            ++take_k;
        }
        if (take_k == 0) take_k = eq_k;   // nothing reaches top_p: all of them
        const float R = r * cum;
        // The chosen value: largest bits bc >= bk with sum_ge(bc) >= R; then
        // the m-th equal element (by index) at which the running sum gets there.
        const uint32_t bc = search(bk, R);
        const float pc = __uint_as_float(bc) / sum;
        float acc = sum_ge(bc + 1);
        const int eq_c = bc == bk ? take_k : count_eq(bc);
        int m = 0;
        while (m < eq_c && acc < R) {
            acc += pc;
            ++m;
        }
        int chosen = INT32_MAX;
        if (acc >= R && m >= 1) {
            // the m-th element in index order whose e has bits bc
            int own = 0;
            for (int i = i0; i < i1; ++i) own += __float_as_uint(lg[i]) == bc;
            const int before = block_excl_scan<NT, int>(own, ipart);
            int hit = INT32_MAX;
            if (before < m && m <= before + own) {
                int c = before;
                for (int i = i0; i < i1; ++i)
                    if (__float_as_uint(lg[i]) == bc && ++c == m) {
                        hit = i;
                        break;
                    }
            }
            chosen = block_min_i<NT>(hit, ipart);
        } else {
            // no element reached R: the reference keeps idx[0], the largest e
            // (e = expf(0) = 1), the lowest index among equal largest ones
            int best = INT32_MAX;
            for (int i = tid; i < n; i += NT)
                if (lg[i] == 1.0f && i < best) best = i;
            chosen = block_min_i<NT>(best, ipart);
        }
        if (tid == 0) *out = chosen == INT32_MAX ? 0 : chosen;
        return;
    }
    // Plain temperature sampling: the first index whose running sum of p
    // reaches r; the runs' sums are scanned across the CTA in index order.
    float own = 0.0f;
    for (int i = i0; i < i1; ++i) own += lg[i] / sum;
    float acc = block_excl_scan<NT, float>(own, fpart);
    int hit = INT32_MAX;
    for (int i = i0; i < i1; ++i) {
        acc += lg[i] / sum;
        if (acc >= r) {
            hit = i;
            break;
        }
    }
    hit = block_min_i<NT>(hit, ipart);
    if (tid == 0) *out = hit == INT32_MAX ? n - 1 : hit;
}

// Token embeddings of a quantized type become an F32 table at load, as
// pickle_fast_state_init does with pickle_dequant_stream
// (src/pickle_fast.c:1551-1584, src/pickle.c:661-870), with that
// function's expressions, each product and difference rounded once:
//   Q8_0  d * q                  Q4_0  d * (q - 8)
//   Q6_K  d * (sc * q)           Q4_K  (d * sc) * q - dmin * m
// One thread per 32-element block (Q8_0, Q4_0), one warp per 256-element
// block (Q4_K, Q6_K: lane l writes elements l, l + 32, ... of the block).
__device__ __forceinline__ float h2f(const unsigned char* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__global__ void dequant32_kernel(const unsigned char* __restrict__ w, int type, size_t n_blocks, float* __restrict__ out) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks; b += stride) {
        float* o = out + b * 32;
        if (type == T_Q8_0) {
            const unsigned char* blk = w + b * 34;
            const float d = h2f(blk);
            for (int i = 0; i < 32; ++i) o[i] = __fmul_rn(d, (float)(int)(signed char)blk[2 + i]);
        } else {
            const unsigned char* blk = w + b * 18;
            const float d = h2f(blk);
            for (int i = 0; i < 16; ++i) {
                o[i] = __fmul_rn(d, (float)((blk[2 + i] & 0x0F) - 8));
                o[16 + i] = __fmul_rn(d, (float)((blk[2 + i] >> 4) - 8));
            }
        }
    }
}

__global__ void dequant256_kernel(const unsigned char* __restrict__ w, int type, size_t n_blocks,
                                  float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const size_t warps = (size_t)gridDim.x * (blockDim.x >> 5);
    for (size_t b = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps) {
        float* o = out + b * 256;
        if (type == T_Q4_K) {
            // d, dmin, scales[12], qs[128]; element 64c + l (l < 32) is the low
            // nibble of qs[32c + l] with sub-block 2c, 64c + 32 + l the high
            // nibble with sub-block 2c + 1.
            const unsigned char* blk = w + b * 144;
            const float d = h2f(blk), dmin = h2f(blk + 2);
            const unsigned char* sc = blk + 4;
            const unsigned char* qs = blk + 16;
            for (int c = 0; c < 4; ++c) {
                for (int half = 0; half < 2; ++half) {
                    const int j = 2 * c + half;
                    int s, m;
                    if (j < 4) {
                        s = sc[j] & 63;
                        m = sc[j + 4] & 63;
                    } else {
                        s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
                        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
                    }
                    const float d1 = __fmul_rn(d, (float)s), m1 = __fmul_rn(dmin, (float)m);
                    const int q = half ? qs[32 * c + lane] >> 4 : qs[32 * c + lane] & 0x0F;
                    o[64 * c + 32 * half + lane] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
                }
            }
        } else {
            // ql[128], qh[64], int8 scales[16], d; element 128n + 32u + l is
            // (ql nibble | 2 bits of qh) - 32, times scales[(128n + 32u + l) / 16].
            const unsigned char* blk = w + b * 210;
            const unsigned char* ql = blk;
            const unsigned char* qh = blk + 128;
            const signed char* scales = reinterpret_cast<const signed char*>(blk + 192);
            const float d = h2f(blk + 208);
            for (int n = 0; n < 2; ++n) {
                for (int u = 0; u < 4; ++u) {
                    const unsigned char lb = ql[64 * n + lane + 32 * (u & 1)];
                    const int lo = u < 2 ? (lb & 0x0F) : (lb >> 4);
                    const int q = (lo | (((qh[32 * n + lane] >> (2 * u)) & 3) << 4)) - 32;
                    const int i = 128 * n + 32 * u + lane;
                    o[i] = __fmul_rn(d, (float)((int)scales[i / 16] * q));
                }
            }
        }
    }
}

// Launch with programmatic stream serialization: the kernel may be
// scheduled before the previous one in the stream ends, and waits for it
// with griddepcontrol.wait before it reads anything.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), unsigned grid, unsigned block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Float4s per thread for a row of n floats, as a template choice.
int norm_vec(int n) {
    const int per = (n / 4 + kNormThreads - 1) / kNormThreads;
    int v = 1;
    while (v < per) v <<= 1;
    return v;
}

cudaError_t launch_add_rmsnorm(int T, float* x, const float* delta, const float* w, float* xn, int n, float eps,
                               cudaStream_t st) {
    switch (norm_vec(n)) {
        case 1: return launch_pdl(add_rmsnorm_kernel<1>, T, kNormThreads, st, x, delta, w, xn, n, eps);
        case 2: return launch_pdl(add_rmsnorm_kernel<2>, T, kNormThreads, st, x, delta, w, xn, n, eps);
        case 4: return launch_pdl(add_rmsnorm_kernel<4>, T, kNormThreads, st, x, delta, w, xn, n, eps);
        case 8: return launch_pdl(add_rmsnorm_kernel<8>, T, kNormThreads, st, x, delta, w, xn, n, eps);
        default: return launch_pdl(add_rmsnorm_kernel<16>, T, kNormThreads, st, x, delta, w, xn, n, eps);
    }
}

cudaError_t launch_embed_rmsnorm(int T, const int32_t* tok, const void* emb, int f16, int vocab, const float* w,
                                 float* x, float* xn, int n, float eps, int* err, cudaStream_t st) {
    switch (norm_vec(n)) {
        case 1: return launch_pdl(embed_rmsnorm_kernel<1>, T, kNormThreads, st, tok, emb, f16, vocab, w, x, xn, n, eps, err);
        case 2: return launch_pdl(embed_rmsnorm_kernel<2>, T, kNormThreads, st, tok, emb, f16, vocab, w, x, xn, n, eps, err);
        case 4: return launch_pdl(embed_rmsnorm_kernel<4>, T, kNormThreads, st, tok, emb, f16, vocab, w, x, xn, n, eps, err);
        case 8: return launch_pdl(embed_rmsnorm_kernel<8>, T, kNormThreads, st, tok, emb, f16, vocab, w, x, xn, n, eps, err);
        default: return launch_pdl(embed_rmsnorm_kernel<16>, T, kNormThreads, st, tok, emb, f16, vocab, w, x, xn, n, eps, err);
    }
}

// pickle_fast_argmax (src/pickle_fast.c:2186-2194): a scan from index 0 that
// keeps the first strictly larger value. Equivalent parallel form: 0 when
// logits[0] is NaN (nothing compares greater than it); otherwise the first
// index of the largest non-NaN value, and 0 when no value exceeds -inf.
// One CTA per row; each thread scans its strided indices in increasing
// order, then the CTA keeps the larger value, ties going to the lower index.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ logits, int n,
                                                                int32_t* __restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    logits += (size_t)blockIdx.x * n;   // one CTA per row of [rows][n]
    out += blockIdx.x;
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    float best = -INFINITY;
    int bi = INT32_MAX;
    for (int i = threadIdx.x; i < n; i += kArgmaxThreads) {
        const float v = logits[i];
        if (v > best) {
            best = v;
            bi = i;
        }
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi != INT32_MAX && (bi == INT32_MAX || ov > best || (ov == best && oi < bi))) {
            best = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        best = l < kArgmaxThreads / 32 ? sv[l] : -INFINITY;
        bi = l < kArgmaxThreads / 32 ? si[l] : INT32_MAX;
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != INT32_MAX && (bi == INT32_MAX || ov > best || (ov == best && oi < bi))) {
                best = ov;
                bi = oi;
            }
        }
        if (l == 0) *out = (bi == INT32_MAX || isnan(logits[0])) ? 0 : bi;
    }
}

size_t row_bytes_of(int type, int in_n) { return pickle_cuda_matvec_row_bytes(type, in_n); }

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

struct DevTensor {
    int type = -1;
    const void* d = nullptr;
    size_t nbytes = 0;
    const float* rowsc = nullptr;   // the GEMM's row scales, computed at load (quantized types)
};

}  // namespace

// Tensor roles of one layer, in the order of pickle_cuda_model_params_t.layers.
enum { R_ATTN_NORM, R_Q, R_K, R_V, R_O, R_FFN_NORM, R_GATE, R_UP, R_DOWN };

struct pickle_cuda_model {
    int device = 0;
    int NL = 0, HD = 0, ID = 0, H = 0, HK = 0, D = 0, VS = 0, max_seq = 0, max_tok = 0, precision = 0;
    int S = 1;        // cache slots (sequences)
    int rows = 0;     // activation rows: max(max_tok, S)
    float eps = 0;
    pickle_cuda_t* attn = nullptr;
    void* blob = nullptr;            // the uploaded weights (null: caller-owned device pointers)
    float* embd_f32 = nullptr;       // a quantized token_embd, dequantized at load
    float* rowsc = nullptr;          // the GEMM row scales of the quantized matrices
    DevTensor embd, out_norm, out;   // out.d == embd.d when tied
    std::vector<DevTensor> lt;       // [NL][9]
    // Per layer: how many of q, k, v (1..3) form one matrix (same type, rows
    // back to back in memory), and whether gate and up do.
    std::vector<int> qkv_run;
    std::vector<char> gu_fused;
    // activations [max_tok][...] and the GEMM workspace; gate holds
    // [max_tok][2 ID] (the fused gate|up output), qkv1 one token's q|k|v
    float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *ao = nullptr, *proj = nullptr,
          *gate = nullptr, *up = nullptr, *logits = nullptr, *logits2 = nullptr, *qkv1 = nullptr;
    int32_t *tok = nullptr, *ids = nullptr;   // ids: [max_seq + 1]
    int* err = nullptr;
    int32_t* ids_host = nullptr;              // pinned [max_seq + 1]
    void* ws = nullptr;
    size_t ws_bytes = 0;
    void* act_blob = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev = nullptr;
    std::string last_error;
};

namespace {

int fail(pickle_cuda_model* m, int rc, const char* what) {
    if (m) m->last_error = what;
    return rc;
}

// A projection with the model's own (constant) weights.
int mm(pickle_cuda_model* m, const DevTensor& w, const float* x, float* y, int out_n, int in_n, int T,
       cudaStream_t st) {
    return pcu_matmul_ex(w.type, w.d, out_n, in_n, T, x, y, m->ws, m->ws_bytes, st, true, w.rowsc);
}

// How the next id is taken from the last row's logits: pickle_fast_argmax
// when temp <= 0, else pickle_fast_sample_temp with (temp, top_p, seed).
struct Pick {
    float temp = 0.0f, top_p = 0.0f;
    uint32_t seed = 0;
};

cudaError_t launch_pick(const Pick& pk, float* logits, int n, int32_t* out, cudaStream_t st) {
    if (!(pk.temp > 0.0f)) return launch_pdl(argmax_kernel, 1, kArgmaxThreads, st, (const float*)logits, n, out);
    return launch_pdl(sample_kernel, 1, kSampleThreads, st, logits, n, pk.temp, pk.top_p, pk.seed, out);
}

// Where the attention of a pass reads and writes the cache:
//   n == 0: T tokens of cache slot `slot` at positions [pos0, pos0 + T)
//           (slot 0: pickle_cuda_prefill_dev / pickle_cuda_decode_batch_dev,
//           other slots: pickle_cuda_prefill_slot_dev);
//   n > 0:  one token of each of n sequences, sequence i at position
//           pos_dev[i] of slot slot_dev[i] (pickle_cuda_decode_ragged_dev);
//           every row then gets logits and an argmax.
struct Attn {
    int slot = 0;
    int n = 0;
    const int* pos_dev = nullptr;
    const int* slot_dev = nullptr;
    size_t max_pos = 0;
};

// T tokens (device ids at tok_dev) at positions [pos0, pos0 + T), T <= max_tok,
// all layers; when with_logits, the last row's logits go to logits_dev and
// its argmax to next_dev (when non-null). Asynchronous on st.
int run_chunk(pickle_cuda_model* m, const int32_t* tok_dev, int T, size_t pos0, bool with_logits, float* logits_dev,
              int32_t* next_dev, cudaStream_t st, const Pick& pk = Pick(), const Attn& at = Attn()) {
    const int HD = m->HD, ID = m->ID, qd = m->H * m->D, kd = m->HK * m->D;
    const DevTensor* L0 = &m->lt[0];
    if (launch_embed_rmsnorm(T, tok_dev, m->embd.d, m->embd.type == T_F16, m->VS,
                             static_cast<const float*>(L0[R_ATTN_NORM].d), m->x, m->xn, HD, m->eps, m->err,
                             st) != cudaSuccess)
        return fail(m, PICKLE_ERR_DEVICE, "embedding launch failed");
    int rc = PICKLE_OK;
    for (int L = 0; L < m->NL; ++L) {
        const DevTensor* W = &m->lt[(size_t)L * kLayerTensors];
        if (L > 0 && launch_add_rmsnorm(T, m->x, m->proj, static_cast<const float*>(W[R_ATTN_NORM].d), m->xn, HD,
                                        m->eps, st) != cudaSuccess)
            return fail(m, PICKLE_ERR_DEVICE, "norm launch failed");
        // q, k, v. One token: into one q|k|v vector, with the projections
        // that share a matrix in one launch. A prompt: [T][..] each, as the
        // causal prefill reads them.
        float *q = m->q, *k = m->k, *v = m->v;
        if (T == 1) {
            q = m->qkv1;
            k = q + qd;
            v = k + kd;
            const int run = m->qkv_run[L];
            const int rows1 = run == 3 ? qd + 2 * kd : run == 2 ? qd + kd : qd;
            if ((rc = mm(m, W[R_Q], m->xn, q, rows1, HD, 1, st)) != PICKLE_OK) return fail(m, rc, "q projection");
            if (run < 2 && (rc = mm(m, W[R_K], m->xn, k, kd, HD, 1, st)) != PICKLE_OK)
                return fail(m, rc, "k projection");
            if (run < 3 && (rc = mm(m, W[R_V], m->xn, v, kd, HD, 1, st)) != PICKLE_OK)
                return fail(m, rc, "v projection");
        } else {
            if ((rc = mm(m, W[R_Q], m->xn, q, qd, HD, T, st)) != PICKLE_OK) return fail(m, rc, "q projection");
            if ((rc = mm(m, W[R_K], m->xn, k, kd, HD, T, st)) != PICKLE_OK) return fail(m, rc, "k projection");
            if ((rc = mm(m, W[R_V], m->xn, v, kd, HD, T, st)) != PICKLE_OK) return fail(m, rc, "v projection");
        }
        if (at.n > 0)
            rc = pickle_cuda_decode_ragged_dev(m->attn, L, at.n, at.pos_dev, at.slot_dev, at.max_pos, q, k, v, m->ao,
                                               st);
        else if (at.slot == 0)
            rc = T == 1 ? pickle_cuda_decode_batch_dev(m->attn, L, 1, pos0, q, k, v, m->ao, st)
                        : pickle_cuda_prefill_dev(m->attn, L, 1, pos0, (size_t)T, q, k, v, m->ao, m->precision, st);
        else
            rc = pickle_cuda_prefill_slot_dev(m->attn, L, at.slot, pos0, (size_t)T, q, k, v, m->ao,
                                              T == 1 ? PICKLE_CUDA_PREFILL_F32 : m->precision, st);
        if (rc != PICKLE_OK) return fail(m, rc, pickle_cuda_last_error(m->attn));
        if ((rc = mm(m, W[R_O], m->ao, m->proj, HD, qd, T, st)) != PICKLE_OK) return fail(m, rc, "output projection");
        if (launch_add_rmsnorm(T, m->x, m->proj, static_cast<const float*>(W[R_FFN_NORM].d), m->xn, HD, m->eps,
                               st) != cudaSuccess)
            return fail(m, PICKLE_ERR_DEVICE, "norm launch failed");
        // gate and up: one [T][2 ID] output when they share a matrix, else
        // [T][ID] each; act goes to the up buffer.
        long long up_off, ld;
        if (m->gu_fused[L]) {
            if ((rc = mm(m, W[R_GATE], m->xn, m->gate, 2 * ID, HD, T, st)) != PICKLE_OK)
                return fail(m, rc, "gate/up projection");
            up_off = ID;
            ld = 2LL * ID;
        } else {
            if ((rc = mm(m, W[R_GATE], m->xn, m->gate, ID, HD, T, st)) != PICKLE_OK)
                return fail(m, rc, "gate projection");
            if ((rc = mm(m, W[R_UP], m->xn, m->up, ID, HD, T, st)) != PICKLE_OK) return fail(m, rc, "up projection");
            up_off = m->up - m->gate;
            ld = ID;
        }
        const size_t n_act = (size_t)T * ID;
        const unsigned blocks = (unsigned)((n_act + 255) / 256 < 148 * 8 ? (n_act + 255) / 256 : 148 * 8);
        if (launch_pdl(swiglu_kernel, blocks, 256, st, m->gate, up_off, ld, ID, T, m->up) != cudaSuccess)
            return fail(m, PICKLE_ERR_DEVICE, "swiglu launch failed");
        if ((rc = mm(m, W[R_DOWN], m->up, m->proj, HD, ID, T, st)) != PICKLE_OK) return fail(m, rc, "down projection");
    }
    // A chunk before the last one leaves only its cache rows behind.
    if (!with_logits) return PICKLE_OK;
    if (at.n > 0) {
        // One token of each sequence: every row's logits and argmax.
        if (launch_add_rmsnorm(T, m->x, m->proj, static_cast<const float*>(m->out_norm.d), m->xn, HD, m->eps, st) !=
            cudaSuccess)
            return fail(m, PICKLE_ERR_DEVICE, "norm launch failed");
        if ((rc = mm(m, m->out, m->xn, logits_dev, m->VS, HD, T, st)) != PICKLE_OK)
            return fail(m, rc, "output projection (lm_head)");
        if (next_dev && launch_pdl(argmax_kernel, (unsigned)T, kArgmaxThreads, st, (const float*)logits_dev, m->VS,
                                   next_dev) != cudaSuccess)
            return fail(m, PICKLE_ERR_DEVICE, "argmax launch failed");
        return PICKLE_OK;
    }
    // Last token only: x += down; xn = rmsnorm(x, output_norm); logits.
    const size_t last = (size_t)(T - 1) * HD;
    if (launch_add_rmsnorm(1, m->x + last, m->proj + last, static_cast<const float*>(m->out_norm.d), m->xn + last, HD,
                           m->eps, st) != cudaSuccess)
        return fail(m, PICKLE_ERR_DEVICE, "norm launch failed");
    if ((rc = mm(m, m->out, m->xn + last, logits_dev, m->VS, HD, 1, st)) != PICKLE_OK)
        return fail(m, rc, "output projection (lm_head)");
    if (next_dev && launch_pick(pk, logits_dev, m->VS, next_dev, st) != cudaSuccess)
        return fail(m, PICKLE_ERR_DEVICE, "argmax / sampler launch failed");
    return PICKLE_OK;
}

// n tokens already on the device, chunked by max_tok; only the last chunk
// computes logits.
int run_tokens(pickle_cuda_model* m, const int32_t* tok_dev, size_t n, size_t pos0, float* logits_dev,
               int32_t* next_dev, cudaStream_t st) {
    for (size_t c0 = 0; c0 < n; c0 += (size_t)m->max_tok) {
        const int T = (int)(n - c0 < (size_t)m->max_tok ? n - c0 : (size_t)m->max_tok);
        const bool last = c0 + (size_t)T == n;
        const int rc = run_chunk(m, tok_dev + c0, T, pos0 + c0, last, logits_dev, next_dev, st);
        if (rc != PICKLE_OK) return rc;
    }
    return PICKLE_OK;
}

// Waits for the stream, then collects the device error words: the model's
// (token ids out of range), the attention handle's (bounded waits, device
// argument checks) and the matvec's (bounded waits).
int finish(pickle_cuda_model* m, cudaStream_t st) {
    if (cudaStreamSynchronize(st) != cudaSuccess) return fail(m, PICKLE_ERR_DEVICE, "stream synchronize failed");
    int e = 0;
    if (cudaMemcpy(&e, m->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(m, PICKLE_ERR_DEVICE, "error word read failed");
    if (e) {
        cudaMemset(m->err, 0, sizeof(int));
        return fail(m, PICKLE_ERR_RANGE, "token id outside [0, vocab) on the device");
    }
    int rc = pickle_cuda_sync(m->attn, st);
    if (rc != PICKLE_OK) return fail(m, rc, pickle_cuda_last_error(m->attn));
    int code = 0;
    if (pickle_cuda_matvec_take_error(m->device, &code) != PICKLE_OK || code)
        return fail(m, PICKLE_ERR_DEVICE, "projection kernel gave up waiting");
    return PICKLE_OK;
}

void free_model(pickle_cuda_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->attn) pickle_cuda_free(m->attn);
    cudaFree(m->blob);
    cudaFree(m->embd_f32);
    cudaFree(m->rowsc);
    cudaFree(m->act_blob);
    cudaFree(m->ws);
    if (m->ids_host) cudaFreeHost(m->ids_host);
    if (m->ev) cudaEventDestroy(m->ev);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int check_matrix(const pickle_cuda_tensor_t& t, int out_n, int in_n, bool on_dev) {
    if (!t.data) return PICKLE_ERR_ARCH;
    const size_t rb = row_bytes_of(t.type, in_n);
    if (t.type != T_F32 && t.type != T_F16 && t.type != T_Q4_0 && t.type != T_Q8_0 && t.type != T_Q4_K &&
        t.type != T_Q6_K)
        return PICKLE_ERR_TYPE;
    if (rb == 0 || t.nbytes != rb * (size_t)out_n) return PICKLE_ERR_ARG;
    if (on_dev && (uintptr_t)t.data % 16) return PICKLE_ERR_ARG;
    return PICKLE_OK;
}

int check_vector(const pickle_cuda_tensor_t& t, int n, bool on_dev) {
    if (!t.data) return PICKLE_ERR_ARCH;
    if (t.type != T_F32) return PICKLE_ERR_TYPE;
    if (t.nbytes != (size_t)n * 4) return PICKLE_ERR_ARG;
    if (on_dev && (uintptr_t)t.data % 16) return PICKLE_ERR_ARG;
    return PICKLE_OK;
}

}  // namespace

extern "C" PICKLE_CUDA_API int pickle_cuda_model_load(const pickle_cuda_model_params_t* p, int device,
                                                      pickle_cuda_model_t** out) {
    if (!p || !out) return PICKLE_ERR_ARG;
    *out = nullptr;
    if (p->n_layers < 1 || p->hidden_dim < 4 || p->hidden_dim % 4 || p->intermediate_dim < 4 ||
        p->intermediate_dim % 4 || p->n_heads < 1 || p->n_kv_heads < 1 || p->n_heads % p->n_kv_heads ||
        p->head_dim < 4 || p->head_dim % 4 || p->vocab_size < 1 || p->max_seq < 1 || p->max_tokens < 1 ||
        p->hidden_dim > 4 * kMaxNormVec * kNormThreads || p->n_seqs < 0 || p->n_seqs > 4096 ||
        !(p->rms_eps >= 0.0f) || !p->layers ||
        (p->prefill_precision != PICKLE_CUDA_PREFILL_F32 && p->prefill_precision != PICKLE_CUDA_PREFILL_BF16))
        return PICKLE_ERR_ARG;
    const bool on_dev = p->weights_on_device != 0;
    const int HD = p->hidden_dim, ID = p->intermediate_dim, qd = p->n_heads * p->head_dim,
              kd = p->n_kv_heads * p->head_dim;
    // Shapes and types, as pickle_fast_state_init finds them (src/pickle_fast.c:1530-1633).
    const pickle_cuda_tensor_t& E = p->token_embd;
    if (!E.data) return PICKLE_ERR_ARCH;
    if (E.type != T_F32 && E.type != T_F16 && E.type != T_Q4_0 && E.type != T_Q8_0 && E.type != T_Q4_K &&
        E.type != T_Q6_K)
        return PICKLE_ERR_TYPE;
    const bool e_quant = E.type != T_F32 && E.type != T_F16;
    if (row_bytes_of(E.type, HD) == 0 || E.nbytes != (size_t)p->vocab_size * row_bytes_of(E.type, HD))
        return PICKLE_ERR_ARG;
    int rc;
    if (p->output_norm.data && (rc = check_vector(p->output_norm, HD, on_dev)) != PICKLE_OK) return rc;
    if (p->output.data && (rc = check_matrix(p->output, p->vocab_size, HD, on_dev)) != PICKLE_OK) return rc;
    for (int L = 0; L < p->n_layers; ++L) {
        const pickle_cuda_tensor_t* t = p->layers + (size_t)L * kLayerTensors;
        if ((rc = check_vector(t[R_ATTN_NORM], HD, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_vector(t[R_FFN_NORM], HD, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_matrix(t[R_Q], qd, HD, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_matrix(t[R_K], kd, HD, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_matrix(t[R_V], kd, HD, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_matrix(t[R_O], HD, qd, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_matrix(t[R_GATE], ID, HD, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_matrix(t[R_UP], ID, HD, on_dev)) != PICKLE_OK) return rc;
        if ((rc = check_matrix(t[R_DOWN], HD, ID, on_dev)) != PICKLE_OK) return rc;
    }
    if (on_dev && (uintptr_t)E.data % 16) return PICKLE_ERR_ARG;

    pickle_cuda_model* m = new (std::nothrow) pickle_cuda_model();
    if (!m) return PICKLE_ERR_MEMORY;
    m->device = device;
    m->NL = p->n_layers; m->HD = HD; m->ID = ID; m->H = p->n_heads; m->HK = p->n_kv_heads; m->D = p->head_dim;
    m->VS = p->vocab_size; m->max_seq = p->max_seq; m->max_tok = p->max_tokens; m->precision = p->prefill_precision;
    m->S = p->n_seqs > 0 ? p->n_seqs : 1;
    m->rows = m->max_tok > m->S ? m->max_tok : m->S;
    m->eps = p->rms_eps;
    if (cudaSetDevice(device) != cudaSuccess) { free_model(m); return PICKLE_ERR_DEVICE; }

    // Attention block state: the device KV cache and RoPE table.
    pickle_cuda_params_t ap{};
    ap.n_layers = p->n_layers; ap.n_heads = p->n_heads; ap.n_kv_heads = p->n_kv_heads; ap.head_dim = p->head_dim;
    ap.max_seq = p->max_seq; ap.half = p->head_dim / 2 < 64 ? p->head_dim / 2 : 64;
    ap.rope_inv_freq = p->rope_inv_freq; ap.rope_theta = p->rope_theta; ap.n_seqs = m->S; ap.rope_len = 0;
    if ((rc = pickle_cuda_init(&ap, device, &m->attn)) != PICKLE_OK) { free_model(m); return rc; }

    // Weights: one allocation, uploaded once, every tensor 256-byte aligned
    // except that k follows q, v follows k and up follows gate with no gap
    // when they have the same type (and the previous one's size is a
    // multiple of 16 bytes): such a run is one [rows][in] matrix, and a
    // decode step projects it in one launch.
    std::vector<const pickle_cuda_tensor_t*> all;
    if (!e_quant) all.push_back(&p->token_embd);
    if (p->output_norm.data) all.push_back(&p->output_norm);
    if (p->output.data) all.push_back(&p->output);
    const size_t lbase = all.size();
    for (size_t i = 0; i < (size_t)p->n_layers * kLayerTensors; ++i) all.push_back(p->layers + i);
    auto packs = [&](size_t i) {
        if (i < lbase) return false;
        const int role = (int)((i - lbase) % kLayerTensors);
        if (role != R_K && role != R_V && role != R_UP) return false;
        if (role == R_V && !(all[i - 1]->type == all[i - 2]->type && all[i - 2]->nbytes % 16 == 0)) return false;
        return all[i]->type == all[i - 1]->type && all[i - 1]->nbytes % 16 == 0;
    };
    std::vector<const void*> where(all.size());
    if (on_dev) {
        for (size_t i = 0; i < all.size(); ++i) where[i] = all[i]->data;
    } else {
        std::vector<size_t> off(all.size());
        size_t total = 0;
        for (size_t i = 0; i < all.size(); ++i) {
            off[i] = i > 0 && packs(i) ? off[i - 1] + all[i - 1]->nbytes : align256(total);
            total = off[i] + all[i]->nbytes;
        }
        if (cudaMalloc(&m->blob, align256(total)) != cudaSuccess) { free_model(m); return PICKLE_ERR_MEMORY; }
        for (size_t i = 0; i < all.size(); ++i) {
            char* dst = static_cast<char*>(m->blob) + off[i];
            if (cudaMemcpy(dst, all[i]->data, all[i]->nbytes, cudaMemcpyHostToDevice) != cudaSuccess) {
                free_model(m);
                return PICKLE_ERR_DEVICE;
            }
            where[i] = dst;
        }
    }
    size_t wi = 0;
    if (!e_quant) {
        m->embd = {E.type, where[wi++], E.nbytes};
    } else {
        // The F32 table the reference builds at state init; the raw bytes
        // are only needed until it is built.
        const void* raw = E.data;
        void* tmp = nullptr;
        const size_t n_el = (size_t)p->vocab_size * HD;
        bool ok = cudaMalloc((void**)&m->embd_f32, n_el * 4) == cudaSuccess;
        if (ok && !on_dev) {
            ok = cudaMalloc(&tmp, E.nbytes) == cudaSuccess &&
                 cudaMemcpy(tmp, E.data, E.nbytes, cudaMemcpyHostToDevice) == cudaSuccess;
            raw = tmp;
        }
        if (ok) {
            const unsigned char* w = static_cast<const unsigned char*>(raw);
            if (E.type == T_Q8_0 || E.type == T_Q4_0)
                dequant32_kernel<<<148 * 8, 256>>>(w, E.type, n_el / 32, m->embd_f32);
            else
                dequant256_kernel<<<148 * 8, 256>>>(w, E.type, n_el / 256, m->embd_f32);
            ok = cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
        }
        cudaFree(tmp);
        if (!ok) { free_model(m); return PICKLE_ERR_DEVICE; }
        m->embd = {T_F32, m->embd_f32, n_el * 4};
    }
    m->out_norm = p->output_norm.data ? DevTensor{T_F32, where[wi++], p->output_norm.nbytes} : DevTensor{};
    // A model without output.weight (or with tied embeddings) projects with
    // token_embd (src/pickle_fast.c:2142-2166).
    m->out = p->output.data ? DevTensor{p->output.type, where[wi++], p->output.nbytes} : m->embd;
    m->lt.resize((size_t)p->n_layers * kLayerTensors);
    for (size_t i = 0; i < m->lt.size(); ++i) m->lt[i] = {p->layers[i].type, where[wi++], p->layers[i].nbytes};
    auto follows = [](const DevTensor& a, const DevTensor& b) {   // b continues matrix a
        return a.type == b.type && static_cast<const char*>(a.d) + a.nbytes == static_cast<const char*>(b.d);
    };
    // The GEMM's per-row weight scales, once: the weights never change. One
    // array, each tensor's rows after the previous one's, so that a fused
    // gate|up matrix finds its rows' scales back to back too.
    {
        struct Job { DevTensor* t; int rows, in; };
        std::vector<Job> jobs;
        const int rows_of[kLayerTensors] = {0, qd, kd, kd, HD, 0, ID, ID, HD};
        const int in_of[kLayerTensors] = {0, HD, HD, HD, qd, 0, HD, HD, ID};
        auto quant = [](int t) { return t == T_Q4_0 || t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K; };
        for (int L = 0; L < p->n_layers; ++L)
            for (int r = 0; r < kLayerTensors; ++r) {
                DevTensor* t = &m->lt[(size_t)L * kLayerTensors + r];
                if (rows_of[r] && quant(t->type)) jobs.push_back({t, rows_of[r], in_of[r]});
            }
        if (p->output.data && quant(m->out.type)) jobs.push_back({&m->out, p->vocab_size, HD});
        size_t total = 0;
        for (auto& e : jobs) total += (size_t)e.rows;
        if (total > 0) {
            if (cudaMalloc((void**)&m->rowsc, total * 4) != cudaSuccess) { free_model(m); return PICKLE_ERR_MEMORY; }
            size_t off = 0;
            for (auto& e : jobs) {
                if (pcu_matmul_rowscale(e.t->type, e.t->d, e.rows, e.in, m->rowsc + off, nullptr) != PICKLE_OK) {
                    free_model(m);
                    return PICKLE_ERR_DEVICE;
                }
                e.t->rowsc = m->rowsc + off;
                off += (size_t)e.rows;
            }
            if (cudaDeviceSynchronize() != cudaSuccess) { free_model(m); return PICKLE_ERR_DEVICE; }
        }
    }
    m->qkv_run.assign(p->n_layers, 1);
    m->gu_fused.assign(p->n_layers, 0);
    for (int L = 0; L < p->n_layers; ++L) {
        const DevTensor* W = &m->lt[(size_t)L * kLayerTensors];
        if (follows(W[R_Q], W[R_K])) m->qkv_run[L] = follows(W[R_K], W[R_V]) ? 3 : 2;
        m->gu_fused[L] = follows(W[R_GATE], W[R_UP]);
    }

    // Activations for max_tok rows.
    const size_t T = (size_t)m->rows;
    const size_t sizes[] = {T * HD * 4, T * HD * 4, T * qd * 4, T * kd * 4, T * kd * 4, T * qd * 4, T * HD * 4,
                            2 * T * ID * 4, T * ID * 4, (size_t)m->VS * 4, (size_t)m->VS * 4, T * 4,
                            ((size_t)m->max_seq + 1) * 4, 256, (size_t)(qd + 2 * kd) * 4};
    size_t total = 0;
    for (size_t s : sizes) total += align256(s);
    if (cudaMalloc(&m->act_blob, total) != cudaSuccess) { free_model(m); return PICKLE_ERR_MEMORY; }
    char* a = static_cast<char*>(m->act_blob);
    void** dst[] = {(void**)&m->x, (void**)&m->xn, (void**)&m->q, (void**)&m->k, (void**)&m->v, (void**)&m->ao,
                    (void**)&m->proj, (void**)&m->gate, (void**)&m->up, (void**)&m->logits, (void**)&m->logits2, (void**)&m->tok,
                    (void**)&m->ids, (void**)&m->err, (void**)&m->qkv1};
    for (size_t i = 0; i < sizeof(sizes) / sizeof(sizes[0]); ++i) {
        *dst[i] = a;
        a += align256(sizes[i]);
    }
    if (cudaMemset(m->err, 0, sizeof(int)) != cudaSuccess) { free_model(m); return PICKLE_ERR_DEVICE; }
    const int shapes[][2] = {{qd, HD}, {kd, HD}, {HD, qd}, {ID, HD}, {2 * ID, HD}, {HD, ID}, {p->vocab_size, HD}};
    // Every row count a pass can have: the split-K partials do not grow with it.
    const int counts[] = {m->rows, 128, 64, 32, 8, 2};
    for (auto& s : shapes)
        for (int c : counts) {
            if (c > m->rows) continue;
            const size_t b = pickle_cuda_matmul_workspace(s[0], s[1], c);
            if (b > m->ws_bytes) m->ws_bytes = b;
        }
    if (cudaMalloc(&m->ws, m->ws_bytes) != cudaSuccess) { free_model(m); return PICKLE_ERR_MEMORY; }
    if (cudaHostAlloc((void**)&m->ids_host, ((size_t)m->max_seq + 1) * 4, cudaHostAllocDefault) != cudaSuccess ||
        cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&m->ev, cudaEventDisableTiming) != cudaSuccess) {
        free_model(m);
        return PICKLE_ERR_DEVICE;
    }
    *out = m;
    return PICKLE_OK;
}

extern "C" PICKLE_CUDA_API void pickle_cuda_model_free(pickle_cuda_model_t* m) { free_model(m); }

extern "C" PICKLE_CUDA_API pickle_cuda_t* pickle_cuda_model_attn(pickle_cuda_model_t* m) {
    return m ? m->attn : nullptr;
}

extern "C" PICKLE_CUDA_API const char* pickle_cuda_model_last_error(pickle_cuda_model_t* m) {
    return m ? m->last_error.c_str() : "null model";
}

extern "C" PICKLE_CUDA_API int pickle_cuda_forward_slot(pickle_cuda_model_t* m, int slot, const int32_t* tokens,
                                                        size_t n_tokens, float* out_logits, size_t* kv_pos) {
    if (!m || !tokens || !out_logits || !kv_pos || n_tokens == 0) return PICKLE_ERR_ARG;
    if (slot < 0 || slot >= m->S) return fail(m, PICKLE_ERR_RANGE, "cache slot outside [0, n_seqs)");
    Attn at;
    at.slot = slot;
    if (cudaSetDevice(m->device) != cudaSuccess) return PICKLE_ERR_DEVICE;
    const size_t pos0 = *kv_pos;
    // The reference stops at the first token outside [0, vocab) or at a
    // position >= max_seq (src/pickle_fast.c:1881-1885) and leaves kv_pos
    // where it was; checking them all first gives the same status and kv_pos.
    for (size_t i = 0; i < n_tokens; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->VS) return fail(m, PICKLE_ERR_RANGE, "token id outside [0, vocab)");
    if (pos0 + n_tokens > (size_t)m->max_seq) return fail(m, PICKLE_ERR_RANGE, "position >= max_seq");
    cudaStream_t st = m->stream;
    for (size_t c0 = 0; c0 < n_tokens; c0 += (size_t)m->max_tok) {
        const size_t T = n_tokens - c0 < (size_t)m->max_tok ? n_tokens - c0 : (size_t)m->max_tok;
        if (cudaMemcpyAsync(m->tok, tokens + c0, T * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return fail(m, PICKLE_ERR_DEVICE, "token upload failed");
        const bool last = c0 + T == n_tokens;
        const int rc = run_chunk(m, m->tok, (int)T, pos0 + c0, last, m->logits, nullptr, st, Pick(), at);
        if (rc != PICKLE_OK) return rc;
        if (!last && cudaStreamSynchronize(st) != cudaSuccess)   // m->tok is reused by the next chunk
            return fail(m, PICKLE_ERR_DEVICE, "stream synchronize failed");
    }
    if (cudaMemcpyAsync(out_logits, m->logits, (size_t)m->VS * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return fail(m, PICKLE_ERR_DEVICE, "logits download failed");
    const int rc = finish(m, st);
    if (rc != PICKLE_OK) return rc;
    *kv_pos = pos0 + n_tokens;
    return PICKLE_OK;
}

extern "C" PICKLE_CUDA_API int pickle_cuda_forward(pickle_cuda_model_t* m, const int32_t* tokens, size_t n_tokens,
                                                   float* out_logits, size_t* kv_pos) {
    return pickle_cuda_forward_slot(m, 0, tokens, n_tokens, out_logits, kv_pos);
}

extern "C" PICKLE_CUDA_API int pickle_cuda_forward_batch_dev(pickle_cuda_model_t* m, int n, const int32_t* tokens_dev,
                                                             const int* pos_dev, const int* slot_dev, size_t max_pos,
                                                             float* logits_dev, int32_t* next_dev, void* stream) {
    if (!m || !tokens_dev || !pos_dev || !slot_dev || !logits_dev || n < 1) return PICKLE_ERR_ARG;
    if (n > m->S) return fail(m, PICKLE_ERR_RANGE, "more sequences than cache slots");
    if ((uintptr_t)logits_dev % 16 || (n > 1 && m->VS % 4)) return fail(m, PICKLE_ERR_ARG, "logits rows unaligned");
    if (max_pos >= (size_t)m->max_seq) return fail(m, PICKLE_ERR_RANGE, "position >= max_seq");
    if (cudaSetDevice(m->device) != cudaSuccess) return PICKLE_ERR_DEVICE;
    Attn at;
    at.n = n;
    at.pos_dev = pos_dev;
    at.slot_dev = slot_dev;
    at.max_pos = max_pos;
    return run_chunk(m, tokens_dev, n, 0, true, logits_dev, next_dev, static_cast<cudaStream_t>(stream), Pick(), at);
}

extern "C" PICKLE_CUDA_API int pickle_cuda_forward_dev(pickle_cuda_model_t* m, const int32_t* tokens_dev,
                                                       size_t n_tokens, size_t pos0, float* logits_dev,
                                                       int32_t* next_dev, void* stream) {
    if (!m || !tokens_dev || !logits_dev || n_tokens == 0) return PICKLE_ERR_ARG;
    if ((uintptr_t)logits_dev % 16) return PICKLE_ERR_ARG;
    if (pos0 + n_tokens > (size_t)m->max_seq) return fail(m, PICKLE_ERR_RANGE, "position >= max_seq");
    if (cudaSetDevice(m->device) != cudaSuccess) return PICKLE_ERR_DEVICE;
    return run_tokens(m, tokens_dev, n_tokens, pos0, logits_dev, next_dev, static_cast<cudaStream_t>(stream));
}

extern "C" PICKLE_CUDA_API int pickle_cuda_argmax_dev(const float* logits, int n, int32_t* out, void* stream) {
    if (!logits || !out || n < 1) return PICKLE_ERR_ARG;
    argmax_kernel<<<1, kArgmaxThreads, 0, static_cast<cudaStream_t>(stream)>>>(logits, n, out);
    return cudaGetLastError() == cudaSuccess ? PICKLE_OK : PICKLE_ERR_DEVICE;
}

extern "C" PICKLE_CUDA_API int pickle_cuda_model_sync(pickle_cuda_model_t* m, void* stream) {
    if (!m) return PICKLE_ERR_ARG;
    if (cudaSetDevice(m->device) != cudaSuccess) return PICKLE_ERR_DEVICE;
    return finish(m, static_cast<cudaStream_t>(stream));
}

extern "C" PICKLE_CUDA_API int pickle_cuda_generate_sampled(pickle_cuda_model_t* m, const int32_t* prompt,
                                                            size_t n_prompt, int n_gen, int eos_id, float temp,
                                                            float top_p, uint32_t seed, int32_t* out_ids, int* n_out,
                                                            float* last_logits, size_t* kv_pos) {
    if (!m || !prompt || n_prompt == 0 || n_gen < 0 || (n_gen > 0 && !out_ids) || !n_out || !kv_pos)
        return PICKLE_ERR_ARG;
    *n_out = 0;
    if (cudaSetDevice(m->device) != cudaSuccess) return PICKLE_ERR_DEVICE;
    for (size_t i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->VS) return fail(m, PICKLE_ERR_RANGE, "token id outside [0, vocab)");
    size_t pos = *kv_pos;
    if (pos + n_prompt > (size_t)m->max_seq) return fail(m, PICKLE_ERR_RANGE, "position >= max_seq");
    cudaStream_t st = m->stream;
    // The prompt in one forward (src/pickle_host.c:473-475); its argmax is id 0.
    for (size_t c0 = 0; c0 < n_prompt; c0 += (size_t)m->max_tok) {
        const size_t T = n_prompt - c0 < (size_t)m->max_tok ? n_prompt - c0 : (size_t)m->max_tok;
        if (cudaMemcpyAsync(m->tok, prompt + c0, T * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return fail(m, PICKLE_ERR_DEVICE, "token upload failed");
        const bool last = c0 + T == n_prompt;
        Pick pk;
        pk.temp = temp;
        pk.top_p = top_p;
        pk.seed = seed;                         // the chat loop's seed + i, i = 0
        const int rc = run_chunk(m, m->tok, (int)T, pos + c0, last, m->logits, m->ids, st, pk);
        if (rc != PICKLE_OK) return rc;
        if (!last && cudaStreamSynchronize(st) != cudaSuccess)   // m->tok is reused by the next chunk
            return fail(m, PICKLE_ERR_DEVICE, "stream synchronize failed");
    }
    pos += n_prompt;
    // The decode loop of pickle_chat_loop (src/pickle_host.c:489-521): id i
    // is the argmax of the current logits (temp <= 0) or their sample with
    // seed + i; the loop stops after an id
    // equal to eos_id, or when the cache is full, and otherwise forwards id i
    // at the next position, whose argmax is id i + 1. The ids stay on the
    // device (ids[i] feeds the next embedding lookup). Without an eos_id the
    // host only enqueues. With one, the host copies id i out before it
    // enqueues the forward of id i and checks it while that forward runs; a
    // forward after the eos id is thrown away: its logits went to the other
    // of two buffers, and the cache row it wrote lies beyond the returned
    // kv_pos.
    const bool eos = eos_id >= 0;
    float* lbuf[2] = {m->logits, m->logits2};
    int cur = 0, done = 0;
    for (int i = 0; i < n_gen; ++i) {
        if (eos && (cudaMemcpyAsync(m->ids_host + i, m->ids + i, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                    cudaEventRecord(m->ev, st) != cudaSuccess))
            return fail(m, PICKLE_ERR_DEVICE, "id download failed");
        const bool full = pos >= (size_t)m->max_seq;
        const int nxt = eos ? cur ^ 1 : cur;
        if (!full) {
            Pick pk;
            pk.temp = temp;
            pk.top_p = top_p;
            pk.seed = seed + (uint32_t)(i + 1);
            const int rc = run_chunk(m, m->ids + i, 1, pos, true, lbuf[nxt], m->ids + i + 1, st, pk);
            if (rc != PICKLE_OK) return rc;
        }
        done = i + 1;
        if (eos) {
            if (cudaEventSynchronize(m->ev) != cudaSuccess) return fail(m, PICKLE_ERR_DEVICE, "event wait failed");
            if (m->ids_host[i] == eos_id) break;
        }
        if (full) break;
        pos += 1;
        cur = nxt;
    }
    int rc = finish(m, st);
    if (rc != PICKLE_OK) return rc;
    if (done > 0 && cudaMemcpy(out_ids, m->ids, (size_t)done * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(m, PICKLE_ERR_DEVICE, "ids download failed");
    if (last_logits &&
        cudaMemcpy(last_logits, lbuf[cur], (size_t)m->VS * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(m, PICKLE_ERR_DEVICE, "logits download failed");
    *n_out = done;
    *kv_pos = pos;
    return PICKLE_OK;
}

extern "C" PICKLE_CUDA_API int pickle_cuda_generate(pickle_cuda_model_t* m, const int32_t* prompt, size_t n_prompt,
                                                    int n_gen, int eos_id, int32_t* out_ids, int* n_out,
                                                    float* last_logits, size_t* kv_pos) {
    return pickle_cuda_generate_sampled(m, prompt, n_prompt, n_gen, eos_id, 0.0f, 0.0f, 0u, out_ids, n_out,
                                        last_logits, kv_pos);
}

extern "C" PICKLE_CUDA_API int pickle_cuda_sample_dev(float* logits, int n, float temp, float top_p, uint32_t seed,
                                                      int32_t* out, void* stream) {
    if (!logits || !out || n < 1) return PICKLE_ERR_ARG;
    Pick pk;
    pk.temp = temp;
    pk.top_p = top_p;
    pk.seed = seed;
    return launch_pick(pk, logits, n, out, static_cast<cudaStream_t>(stream)) == cudaSuccess ? PICKLE_OK
                                                                                              : PICKLE_ERR_DEVICE;
}
