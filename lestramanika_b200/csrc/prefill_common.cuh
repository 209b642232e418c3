// prefill_common.cuh - producer stage of batched causal prefill and the
// log-sum-exp merge of partial attention triples.
//
// The reference prefills token by token (lee-muriithi-kingori/lestramanika
// src/pickle_fast.c:1881, src/pickle_host.c:473): for each prompt token it
// rotates q/k (:1910-1936), appends k/v (:1938-1944) and attends over
// [0, pos]. Batched prefill splits that into one producer launch for all T
// tokens (this file) and one attention launch.
#pragma once
#include "pcu_common.cuh"
#include "decode_splitkv.cuh"

// Rotate the T new tokens of every sequence: q -> q_rot (F32, and BF16 when
// q_bf16 != nullptr), k -> cache rows [pos0, pos0+T) (F32), v -> cache.
// Optional BF16 copies of the rotated k / v rows ([seq][kv_head][T][D])
// feed the tensor-core kernel.
struct RopeAppendArgs {
    const float* q;        // [n_seqs][T][H][D]
    const float* k;        // [n_seqs][T][HK][D]
    const float* v;
    float* q_rot;          // [n_seqs][T][H][D] (may be null)
    float* kc;             // layer K cache
    float* vc;
    long long seq_stride, head_stride;
    const float* sin_tab;
    const float* cos_tab;
    int H, HK, D, half, T;
    long long pos0;
    __nv_bfloat16* q_bf16; // [n_seqs][H][T][D] head-major (may be null)
    __nv_bfloat16* k_bf16; // [n_seqs][HK][T][D]
    __nv_bfloat16* v_bf16; // [n_seqs][HK][T][D]
    float q_prescale;      // multiplies the BF16 q copy (1 for F32 use)
};

__global__ void rope_append_kernel(const RopeAppendArgs a) {
    const int t = blockIdx.x, seq = blockIdx.y;
    griddep_launch_dependents();        // the attention launch may take SM slots as this grid drains
    const long long pos = a.pos0 + t;
    const float* sr = a.sin_tab + (size_t)pos * a.half;
    const float* cr = a.cos_tab + (size_t)pos * a.half;
    const size_t tok = (size_t)seq * a.T + t;
    const float* qt = a.q + tok * a.H * a.D;
    const float* kt = a.k + tok * a.HK * a.D;
    const float* vt = a.v + tok * a.HK * a.D;
    const int nq = a.H * a.D, nk = a.HK * a.D;
    for (int i = threadIdx.x; i < nq; i += blockDim.x) {
        const int h = i / a.D, d = i % a.D;
        const float x = rope_elem(qt + (size_t)h * a.D, d, a.half, sr, cr);
        if (a.q_rot) a.q_rot[tok * nq + i] = x;
        if (a.q_bf16)
            a.q_bf16[(((size_t)seq * a.H + h) * a.T + t) * a.D + d] = __float2bfloat16_rn(x * a.q_prescale);
    }
    for (int i = threadIdx.x; i < nk; i += blockDim.x) {
        const int h = i / a.D, d = i % a.D;
        const float kr = rope_elem(kt + (size_t)h * a.D, d, a.half, sr, cr);
        const float vv = vt[i];
        const size_t row = (size_t)seq * a.seq_stride + (size_t)h * a.head_stride + (size_t)pos * a.D + d;
        a.kc[row] = kr;
        a.vc[row] = vv;
        if (a.k_bf16) {
            const size_t brow = (((size_t)seq * a.HK + h) * a.T + t) * a.D + d;
            a.k_bf16[brow] = __float2bfloat16_rn(kr);
            a.v_bf16[brow] = __float2bfloat16_rn(vv);
        }
    }
}

// Same result as rope_append_kernel with 16-byte accesses: one thread takes a
// rotation pair of float4 chunks (d..d+3, d+half..d+half+3), an unrotated
// float4 chunk past 2*half, or a float4 chunk of v. Needs D % 4 == 0 and
// half % 4 == 0 (checked by the host). One CTA per token.
__global__ void __launch_bounds__(128) rope_append_vec_kernel(const RopeAppendArgs a) {
    const int t = blockIdx.x, seq = blockIdx.y;
    griddep_launch_dependents();        // the attention launch may take SM slots as this grid drains
    const long long pos = a.pos0 + t;
    const int D = a.D, half = a.half;
    const int NP = half / 4, NT = (D - 2 * half) / 4, NU = NP + NT, NC = D / 4;
    const float4* sr = reinterpret_cast<const float4*>(a.sin_tab + (size_t)pos * half);
    const float4* cr = reinterpret_cast<const float4*>(a.cos_tab + (size_t)pos * half);
    const size_t tok = (size_t)seq * a.T + t;
    const int n_q = a.H * NU, n_k = a.HK * NU, n_v = a.HK * NC;
    for (int u = threadIdx.x; u < n_q + n_k + n_v; u += blockDim.x) {
        if (u < n_q + n_k) {
            const bool is_q = u < n_q;
            const int uu = is_q ? u : u - n_q;
            const int h = uu / NU, c = uu % NU;
            const float* row = is_q ? a.q + (tok * a.H + h) * D : a.k + (tok * a.HK + h) * D;
            float4 lo_out, hi_out;
            int d_lo, d_hi = -1;
            if (c < NP) {
                d_lo = 4 * c;
                d_hi = d_lo + half;
                const float4 x0 = *reinterpret_cast<const float4*>(row + d_lo);
                const float4 x1 = *reinterpret_cast<const float4*>(row + d_hi);
                // src/pickle_fast.c:1917-1924: x' = c*x0 - s*x1, x'' = s*x0 + c*x1
                rope_pair4(x0, x1, sr[c], cr[c], lo_out, hi_out);
            } else {
                d_lo = 2 * half + 4 * (c - NP);
                lo_out = *reinterpret_cast<const float4*>(row + d_lo);
            }
            if (is_q) {
                if (a.q_rot) {
                    float* dst = a.q_rot + (tok * a.H + h) * D;
                    *reinterpret_cast<float4*>(dst + d_lo) = lo_out;
                    if (d_hi >= 0) *reinterpret_cast<float4*>(dst + d_hi) = hi_out;
                }
                if (a.q_bf16) {
                    __nv_bfloat16* dst = a.q_bf16 + (((size_t)seq * a.H + h) * a.T + t) * D;
                    *reinterpret_cast<uint2*>(dst + d_lo) = pack_bf16x4(lo_out, a.q_prescale);
                    if (d_hi >= 0) *reinterpret_cast<uint2*>(dst + d_hi) = pack_bf16x4(hi_out, a.q_prescale);
                }
            } else {
                float* dst = a.kc + (size_t)seq * a.seq_stride + (size_t)h * a.head_stride + (size_t)pos * D;
                *reinterpret_cast<float4*>(dst + d_lo) = lo_out;
                if (d_hi >= 0) *reinterpret_cast<float4*>(dst + d_hi) = hi_out;
                if (a.k_bf16) {
                    __nv_bfloat16* bd = a.k_bf16 + (((size_t)seq * a.HK + h) * a.T + t) * D;
                    *reinterpret_cast<uint2*>(bd + d_lo) = pack_bf16x4(lo_out, 1.0f);
                    if (d_hi >= 0) *reinterpret_cast<uint2*>(bd + d_hi) = pack_bf16x4(hi_out, 1.0f);
                }
            }
        } else {
            const int uu = u - n_q - n_k;
            const int h = uu / NC, c = uu % NC;
            const float4 x = *reinterpret_cast<const float4*>(a.v + (tok * a.HK + h) * D + 4 * c);
            float* dst = a.vc + (size_t)seq * a.seq_stride + (size_t)h * a.head_stride + (size_t)pos * D;
            *reinterpret_cast<float4*>(dst + 4 * c) = x;
            if (a.v_bf16) {
                __nv_bfloat16* bd = a.v_bf16 + (((size_t)seq * a.HK + h) * a.T + t) * D;
                *reinterpret_cast<uint2*>(bd + 4 * c) = pack_bf16x4(x, 1.0f);
            }
        }
    }
}

// o = sum_i e^(m_i - M) acc_i / sum_i e^(m_i - M) l_i over n_parts partial
// triples of n_rows rows; one CTA per row, one thread per element. Part i's
// m, l and acc start at m + i*part_stride, l + i*part_stride and
// acc + i*part_stride (floats), with row stride 1 (m, l) and D (acc).
__global__ void lse_merge_kernel(int n_parts, int n_rows, int D, long long part_stride_m,
                                 long long part_stride_acc, const float* __restrict__ m,
                                 const float* __restrict__ l, const float* __restrict__ acc,
                                 float* __restrict__ out) {
    const int row = blockIdx.x;
    float M = -INFINITY;
    for (int i = 0; i < n_parts; ++i) M = fmaxf(M, m[(size_t)i * part_stride_m + row]);
    float L = 0.f;
    for (int i = 0; i < n_parts; ++i) {
        const float mi = m[(size_t)i * part_stride_m + row];
        L += (mi == -INFINITY) ? 0.f : l[(size_t)i * part_stride_m + row] * expf(mi - M);
    }
    const float inv = 1.0f / (L == 0.0f ? 1.0f : L);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float A = 0.f;
        for (int i = 0; i < n_parts; ++i) {
            const float mi = m[(size_t)i * part_stride_m + row];
            if (mi != -INFINITY)
                A = fmaf(expf(mi - M), acc[(size_t)i * part_stride_acc + (size_t)row * D + d], A);
        }
        out[(size_t)row * D + d] = A * inv;
    }
}
