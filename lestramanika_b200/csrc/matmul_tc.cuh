// matmul_tc.cuh - Y = X W^T for many activation rows (the projections of a
// batched prefill), W in its raw GGML blocks, on the sm_100a tensor cores.
//
// The reference runs the forward token by token and multiplies every
// token's activation by the dequantized weights in float
// (pickle_fast_matmul_dispatch, src/pickle_fast.c:1423-1474, called per
// token from the layer loop at :1903-1907, :2112, :2120-2133). Batching the
// prompt turns those T matvecs into one GEMM whose weight tiles are read once
// per 128 tokens. The products keep float accuracy:
//
//   * every weight is dequantized to its float value w as the reference
//     computes it, scaled by a power of two 2^r per weight row (so that the
//     row's largest possible |w| sits below 2^15) and split into f16 hi + lo
//     (w 2^r = hi + lo, 22 significant bits);
//   * every activation row is split the same way, with a power of two per
//     token (xsplit_kernel);
//   * the tensor cores accumulate hi.hi + hi.lo + lo.hi in f32 (the lo.lo
//     term is below f32 rounding); the epilogue removes both powers of two.
//     F16 weights are exact in f16 and need only hi.hi + hi.lo.
//
// Tile = 128 weight rows x BN tokens (BN 128 for prompts, 32 / 64 for decode
// batches). The grid is persistent: at most one CTA per SM, each walking its
// tiles (one tile per CTA when K is split over CTAs):
//   warp 0     one lane streams the raw weight blocks of each 256-element
//              K-block (2-D TMA, 128-row box) and the x hi / lo tiles of each
//              64-element K-step (2-D TMA, 128-byte swizzle); for F16 it loads
//              the weight tile itself the same way;
//   warps 2-5  thread r dequantizes row r of each K-step into the A hi / lo
//              tiles, in the 128-byte-swizzled K-major layout the MMA reads;
//   warp 1     allocates two BN-column TMEM accumulators; one lane issues
//              tcgen05.mma (M = 128, N = BN, K = 16, f16 in, f32 accumulate)
//              into tile i's accumulator while tile i - 1's drains;
//   warps 6-9  read the accumulator rows out of TMEM, store y, and hand the
//              accumulator back to the MMA.
// Every mbarrier wait is bounded (a timeout records an error in g_mv_err and
// the kernel runs on to its end, freeing TMEM). No multicast.
#pragma once
#include "matvec_tc.cuh"

namespace mmtc {

using mvtc::F_F16;
using mvtc::F_Q4_0;
using mvtc::F_Q4_K;
using mvtc::F_Q6_K;
using mvtc::F_Q8_0;

// BN, the token tile (the MMA's N), is 128 for prompts and 32 or 64 for
// small decode batches, whose one token tile would leave most of a
// 128-wide MMA on zero rows.
constexpr int BM = 128, BN = 128, BK = 64, KB = 256;
constexpr int A_STAGES = 2, X_STAGES = 3, RAW_STAGES = 2;
constexpr int TILE = 128 * 128;                       // bytes of one 128 x 64 f16 weight tile
constexpr int THREADS = 320;
inline int bn_for(int n_tok) { return n_tok <= 32 ? 32 : n_tok <= 64 ? 64 : 128; }
// Warps: producer, MMA, DQW dequantizing (one thread per weight row), 4 epilogue.
template <int BNT> struct Cfg {
    static constexpr int DQW = 4;
    static constexpr int THREADS = 32 * (2 + DQW + 4);
};

// Raw weight bytes of one 256-element K-block per row (the TMA box width).
template <int TYPE> struct Raw;
template <> struct Raw<F_F16> { static constexpr int B = 0; };
template <> struct Raw<F_Q4_K> { static constexpr int B = 144; };
template <> struct Raw<F_Q8_0> { static constexpr int B = 272; };   // 8 blocks of 34 bytes
template <> struct Raw<F_Q4_0> { static constexpr int B = 144; };   // 8 blocks of 18 bytes
// One 210-byte block, copied from the 16-byte boundary at or below it: the
// block sits 2 kb mod 16 bytes into the 240-byte window.
template <> struct Raw<F_Q6_K> { static constexpr int B = 240; };

// x coordinate (64-bit words) of K-block kb's window in a raw weight row.
template <int TYPE>
PCU_DEV int raw_x(int kb) {
    if constexpr (TYPE == F_Q6_K) return (kb * 210 - ((2 * kb) & 15)) / 8;
    else return kb * (Raw<TYPE>::B / 8);
}

constexpr int OFF_A = 0;                                  // [AS][hi, lo] weight tiles
template <int TYPE, int BNT> struct Lay {
    static constexpr int XT = BNT * 128;                             // bytes of one BNT x 64 f16 x tile
    static constexpr int XS = Raw<TYPE>::B > 240 && BNT == 128 ? 2 : X_STAGES;   // x ring depth that fits
    static constexpr int AS = A_STAGES;                              // weight-tile (hi, lo) ring
    // Raw weight ring (K-blocks in flight from HBM). A wide token tile has
    // enough tensor work per K-block to hide the latency of two; a narrow
    // one (a decode batch) streams weights and takes as many as fit, up to 6.
    static constexpr int FIXED = XS * 2 * XT + AS * 2 * TILE + 2048;
    static constexpr int RS_FIT = Raw<TYPE>::B ? (232448 - FIXED) / (BM * Raw<TYPE>::B) : RAW_STAGES;
    static constexpr int RS = BNT == 128 || Raw<TYPE>::B == 0 ? RAW_STAGES : RS_FIT > 6 ? 6 : RS_FIT;
    static constexpr int OFF_X = OFF_A + AS * 2 * TILE;              // [XS][hi, lo] x tiles
    static constexpr int OFF_RAW = OFF_X + XS * 2 * XT;              // [RS][BM][Raw::B]
    static constexpr int OFF_BAR = OFF_RAW + RS * BM * Raw<TYPE>::B;
    // RAW_FULL[RS], RAW_EMPTY[RS], A_FULL[AS], A_EMPTY[AS], X_FULL[XS], X_EMPTY[XS],
    // D_FULL[2], ACC_EMPTY[2] (the two TMEM accumulators)
    static constexpr int N_BARS = 2 * RS + 2 * AS + 2 * XS + 4;
    static constexpr int OFF_TMEM = OFF_BAR + N_BARS * 8;
    static constexpr int BYTES = OFF_TMEM + 16 + 1024;     // + alignment slack of the 1024-byte base
    static_assert(BYTES <= 232448, "dynamic shared memory of one CTA on sm_100");
};

// tcgen05 instruction descriptor, kind::f16 with F16 A and B, F32
// accumulate, both K-major, M = 128, N = BNT.
template <int BNT>
__host__ __device__ constexpr uint32_t idesc() { return (1u << 4) | ((uint32_t)(BNT >> 3) << 17) | ((uint32_t)(BM >> 4) << 24); }

// Shared-memory matrix descriptor: 128-byte swizzle, 8-row atoms 1024 bytes apart.
PCU_DEV uint64_t sdesc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                   // leading byte offset (16 bytes; unused with this swizzle)
    d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset
    d |= (uint64_t)1 << 46;                   // sm_100 descriptor version
    d |= (uint64_t)2 << 61;                   // 128-byte swizzle
    return d;
}

PCU_DEV void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc, uint32_t id) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}

PCU_DEV void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

PCU_DEV void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
PCU_DEV void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// Generic-proxy shared-memory writes made visible to the tensor cores.
PCU_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

PCU_DEV void mbar_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

PCU_DEV void tma2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

PCU_DEV void tmem_ld32x(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    #pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Two floats to an f16 pair (a in the low half) and the residual pair.
PCU_DEV void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// --------------------------------------------------------------- pre-passes

// x [n_tok][in_n] (f32) -> xh, xl [n_tok][in_n] (f16) with x * 2^s = xh + xl,
// s per token (its largest |x| just below 2^15); xinv[n] = 2^-s.
__global__ void __launch_bounds__(256) xsplit_kernel(const float* __restrict__ x, int in_n, __half* __restrict__ xh,
                                                     __half* __restrict__ xl, float* __restrict__ xinv) {
    griddep_launch_dependents();
    griddep_wait();                       // x may come from the kernel before
    __shared__ float red[8];
    const int n = blockIdx.x, tid = threadIdx.x;
    const float* xr = x + (size_t)n * in_n;
    float m = 0.f;
    for (int i = 4 * tid; i < in_n; i += 1024) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(xr + i));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = 0.f;
    #pragma unroll
    for (int w = 0; w < 8; ++w) m = fmaxf(m, red[w]);
    int s = 14 - ((int)((__float_as_uint(m) >> 23) & 0xFF) - 127);
    s = max(-126, min(126, s));
    const float sc = __uint_as_float((uint32_t)(127 + s) << 23);
    for (int i = 4 * tid; i < in_n; i += 1024) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(xr + i));
        uint2 h, l;
        split2(q.x * sc, q.y * sc, h.x, l.x);
        split2(q.z * sc, q.w * sc, h.y, l.y);
        *reinterpret_cast<uint2*>(xh + (size_t)n * in_n + i) = h;
        *reinterpret_cast<uint2*>(xl + (size_t)n * in_n + i) = l;
    }
    if (tid == 0) xinv[n] = __uint_as_float((uint32_t)(127 - s) << 23);
}

// Per weight row, 2^r with r chosen so that every |w| of the row is below
// 2^15 after scaling (w 2^r); one warp per row, from the block headers.
template <int TYPE>
__global__ void __launch_bounds__(256) rowscale_kernel(const uint8_t* __restrict__ W, size_t row_bytes, int out_n,
                                                       int in_n, float* __restrict__ rowsc) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= out_n) return;
    const uint8_t* wr = W + (size_t)row * row_bytes;
    float bound = 0.f;
    auto ldh = [&](size_t off) {   // an f16 at a 2-byte aligned offset of the row
        return fabsf(__half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(wr + off)))));
    };
    if constexpr (TYPE == F_Q4_K) {
        // |w| = |d sc q - dmin m| <= 945 |d| + 63 |dmin|
        for (int b = lane; b < in_n / 256; b += 32)
            bound = fmaxf(bound, fmaf(945.f, ldh((size_t)b * 144), 63.f * ldh((size_t)b * 144 + 2)));
    } else if constexpr (TYPE == F_Q8_0) {
        for (int b = lane; b < in_n / 32; b += 32) bound = fmaxf(bound, 128.f * ldh((size_t)b * 34));
    } else if constexpr (TYPE == F_Q4_0) {
        for (int b = lane; b < in_n / 32; b += 32) bound = fmaxf(bound, 8.f * ldh((size_t)b * 18));
    } else if constexpr (TYPE == F_Q6_K) {
        for (int b = lane; b < in_n / 256; b += 32) bound = fmaxf(bound, 4096.f * ldh((size_t)b * 210 + 208));
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) bound = fmaxf(bound, __shfl_xor_sync(0xffffffffu, bound, o));
    int r = 0;
    if (bound > 0.f && bound < 3.0e38f) r = 14 - ((int)((__float_as_uint(bound) >> 23) & 0xFF) - 127);
    r = max(-126, min(126, r));
    if (lane == 0) rowsc[row] = __uint_as_float((uint32_t)(127 + r) << 23);
}

// ---------------------------------------------------------------- dequant

// The 64 weights of K-step ks (elements 64 ks .. 64 ks + 63 of K-block kb)
// of one row, times the row's 2^r; rw = the row's raw window in shared
// memory. Each follows the reference's per-weight expression.
template <int TYPE>
PCU_DEV void dequant_kstep(uint32_t rw, int kb, int ks, float rsc, float (&w)[64]) {
    auto byte_of = [](uint32_t wv, int i) { return (int)((wv >> (8 * i)) & 0xFFu); };
    if constexpr (TYPE == F_Q4_K) {
        // Chunk ks: j < 32 low nibble of qs[32 ks + j] (sub-block 2 ks), else the
        // high nibble of qs[32 ks + j - 32] (sub-block 2 ks + 1); w = d sc q -
        // dmin m with the 6-bit scales and mins of src/pickle_fast.c:368-383.
        const uint4 h = mvtc::lds128(rw);
        const float d = mvtc::h2f_lo(h.x) * rsc, dmin = mvtc::h2f_hi(h.x) * rsc;
        int sc[2], mn[2];
        #pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = 2 * ks + u;
            if (j < 4) {
                sc[u] = byte_of(h.y, j) & 63;
                mn[u] = byte_of(h.z, j) & 63;
            } else {
                sc[u] = (byte_of(h.w, j - 4) & 15) | ((byte_of(h.y, j - 4) >> 6) << 4);
                mn[u] = (byte_of(h.w, j - 4) >> 4) | ((byte_of(h.z, j - 4) >> 6) << 4);
            }
        }
        const float d0 = d * (float)sc[0], m0f = dmin * (float)mn[0];
        const float d1 = d * (float)sc[1], m1f = dmin * (float)mn[1];
        const uint4 qa = mvtc::lds128(rw + 16 + 32 * ks), qb = mvtc::lds128(rw + 32 + 32 * ks);
        const uint32_t wd[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        #pragma unroll
        for (int i = 0; i < 8; ++i)
            #pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint32_t by = (wd[i] >> (8 * b)) & 0xFFu;
                w[4 * i + b] = fmaf(d0, (float)(by & 15u), -m0f);
                w[32 + 4 * i + b] = fmaf(d1, (float)(by >> 4), -m1f);
            }
    } else if constexpr (TYPE == F_Q8_0 || TYPE == F_Q4_0) {
        // Blocks 2 ks and 2 ks + 1 of the K-block (32 elements each): d (f16),
        // then the quants (Q8_0: 32 signed bytes, w = d q; Q4_0: 16 bytes, byte
        // j holds element j in its low nibble and 16 + j in its high one, w =
        // d (q - 8)). The quants are 4-byte aligned in odd blocks only.
        constexpr int BB = TYPE == F_Q8_0 ? 34 : 18;
        #pragma unroll
        for (int u = 0; u < 2; ++u) {
            const uint32_t bp = rw + BB * (2 * ks + u);
            const float d = __half2float(__ushort_as_half((unsigned short)mvtc::ldsu16(bp))) * rsc;
            constexpr int NW = TYPE == F_Q8_0 ? 8 : 4;
            uint32_t q[NW];
            #pragma unroll
            for (int i = 0; i < NW; ++i) q[i] = u ? mvtc::lds32(bp + 2 + 4 * i) : mvtc::lds32_odd2(bp + 2 + 4 * i);
            #pragma unroll
            for (int i = 0; i < NW; ++i)
                #pragma unroll
                for (int b = 0; b < 4; ++b) {
                    if constexpr (TYPE == F_Q8_0) {
                        w[32 * u + 4 * i + b] = d * (float)(int)(signed char)byte_of(q[i], b);
                    } else {
                        const int by = byte_of(q[i], b);
                        w[32 * u + 4 * i + b] = d * (float)((by & 15) - 8);
                        w[32 * u + 16 + 4 * i + b] = d * (float)((by >> 4) - 8);
                    }
                }
        }
    } else if constexpr (TYPE == F_Q6_K) {
        // Element 128n + 32u + l: (ql[64n + l + 32 (u & 1)] low nibble for u < 2,
        // high for u >= 2) | ((qh[32n + l] >> 2u) & 3) << 4, less 32, times
        // d * scales[8n + l/16 + 2u] (src/pickle_fast.c:1084-1257). K-step ks
        // is half n = ks / 2, u = 2 (ks & 1) + (0, 1). The block starts
        // M = 2 kb mod 16 bytes into the window: 4-byte aligned when M % 4 == 0.
        const int n = ks >> 1, hs = 4 * (ks & 1);
        const uint32_t bp = rw + ((2 * kb) & 15);
        const bool al4 = (((2 * kb) & 15) & 3) == 0;
        auto ld4 = [&](uint32_t a) { return al4 ? mvtc::lds32(a) : mvtc::lds32_odd2(a); };
        const float d = __half2float(__ushort_as_half((unsigned short)mvtc::ldsu16(bp + 208))) * rsc;
        float ds[2][2];
        #pragma unroll
        for (int uu = 0; uu < 2; ++uu)
            #pragma unroll
            for (int lh = 0; lh < 2; ++lh) {
                const int u = 2 * (ks & 1) + uu;
                ds[uu][lh] = d * (float)(int)(signed char)mvtc::ldsu8(bp + 192 + 8 * n + lh + 2 * u);
            }
        #pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t qh = ld4(bp + 128 + 32 * n + 4 * i);
            #pragma unroll
            for (int uu = 0; uu < 2; ++uu) {
                const int u = 2 * (ks & 1) + uu;
                const uint32_t ql = ld4(bp + 64 * n + 32 * uu + 4 * i);
                // the four 6-bit quants of bytes 0..3 at once
                const uint32_t q4 = ((ql >> hs) & 0x0F0F0F0Fu) | (((qh >> (2 * u)) & 0x03030303u) << 4);
                #pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int l = 4 * i + b;
                    // quant byte b under the exponent of 2^23: 2^23 + q exactly,
                    // so (2^23 + q) - (2^23 + 32) is (float)(q - 32) exactly
                    const float f = __uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7540u + b));
                    w[32 * uu + l] = ds[uu][l >> 4] * (f - 8388640.0f);
                }
            }
        }
    }
}

// ------------------------------------------------------------------- kernel

template <int TYPE, int BNT>
__global__ void __launch_bounds__(Cfg<BNT>::THREADS, 1)
    matmul_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xh,
                     const __grid_constant__ CUtensorMap tm_xl, int out_n, int in_n, int n_tok,
                     const float* __restrict__ xinv, const float* __restrict__ rowsc, float* __restrict__ y,
                     float* __restrict__ part) {
    using L = Lay<TYPE, BNT>;
    constexpr int XT = L::XT, TMEM_COLS = 2 * BNT;   // two accumulators: tile i+1 while tile i drains
    constexpr uint32_t ID = idesc<BNT>();
    constexpr bool QUANT = TYPE != F_F16;
    constexpr int DQW = Cfg<BNT>::DQW;
    constexpr int A_STAGES = L::AS, OFF_X = L::OFF_X, RAW_STAGES = L::RS;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - smem_u32(smem_raw));
    const uint32_t bar0 = base + L::OFF_BAR;
    const uint32_t RAW_FULL = bar0, RAW_EMPTY = bar0 + 8 * RAW_STAGES, A_FULL = RAW_EMPTY + 8 * RAW_STAGES,
                   A_EMPTY = A_FULL + 8 * A_STAGES, X_FULL = A_EMPTY + 8 * A_STAGES,
                   X_EMPTY = X_FULL + 8 * L::XS, D_FULL = X_EMPTY + 8 * L::XS, ACC_EMPTY = D_FULL + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_TMEM);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Output tiles: a CTA takes tiles blockIdx.x, blockIdx.x + gridDim.x, ...
    // (tile t: weight rows (t % n_mt) * BM, tokens (t / n_mt) * BNT), so the
    // epilogue of one tile overlaps the main loop of the next. Every ring
    // counts its stages on across the tiles.
    const int n_mt = (out_n + BM - 1) / BM;
    const int total = n_mt * ((n_tok + BNT - 1) / BNT);
    // Split K: this CTA takes K-blocks [kb0, kb0 + nkb) of slice blockIdx.z
    // (the host makes every slice non-empty and then gives each CTA one tile).
    const int nkb_all = in_n / KB;
    const int kb0 = (int)blockIdx.z * nkb_all / (int)gridDim.z;
    const int nkb = ((int)blockIdx.z + 1) * nkb_all / (int)gridDim.z - kb0, nks = nkb * (KB / BK);

    if (threadIdx.x == 0) {
        uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
        for (int i = 0; i < RAW_STAGES; ++i) {
            mbar_init(&bars[i], 1);
            mbar_init(&bars[RAW_STAGES + i], DQW);
        }
        for (int i = 0; i < A_STAGES; ++i) {
            mbar_init(&bars[2 * RAW_STAGES + i], QUANT ? DQW : 1);
            mbar_init(&bars[2 * RAW_STAGES + A_STAGES + i], 1);
        }
        for (int i = 0; i < L::XS; ++i) {
            mbar_init(&bars[2 * RAW_STAGES + 2 * A_STAGES + i], 1);
            mbar_init(&bars[2 * RAW_STAGES + 2 * A_STAGES + L::XS + i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars[L::N_BARS - 4 + i], 1);   // D_FULL: the MMAs of a tile are done
            mbar_init(&bars[L::N_BARS - 2 + i], 4);   // ACC_EMPTY: the 4 epilogue warps read it out
        }
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t tmem = *tmem_slot;
    // Launched with programmatic stream serialization: the set-up above ran
    // while the kernel before finished; x, its scales and the row scales may
    // come from that kernel.
    griddep_launch_dependents();
    griddep_wait();

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            #pragma unroll 1
            for (int t = blockIdx.x, it = 0; t < total; t += gridDim.x, ++it) {
            const int m0 = (t % n_mt) * BM, n0 = (t / n_mt) * BNT;
            #pragma unroll 1
            for (int kl0 = 0; kl0 < nkb; ++kl0) {
                const int kb = kb0 + kl0, kl = it * nkb + kl0;   // kl: K-block count across tiles
                if constexpr (QUANT) {
                    const int rs = kl % RAW_STAGES;
                    if (kl >= RAW_STAGES)
                        mvtc::wait_or_flag(RAW_EMPTY + 8 * rs, ((kl / RAW_STAGES) - 1) & 1, PCU_DEVERR_EMPTY_WAIT);
                    mbar_expect(RAW_FULL + 8 * rs, BM * Raw<TYPE>::B);
                    tma2d(base + L::OFF_RAW + rs * BM * Raw<TYPE>::B, &tm_w, raw_x<TYPE>(kb), m0, RAW_FULL + 8 * rs);
                }
                #pragma unroll 1
                for (int ks = 0; ks < KB / BK; ++ks) {
                    const int s = kl * (KB / BK) + ks, k = kb * KB + ks * BK;
                    const int xs = s % L::XS;
                    if (s >= L::XS)
                        mvtc::wait_or_flag(X_EMPTY + 8 * xs, ((s / L::XS) - 1) & 1, PCU_DEVERR_EMPTY_WAIT);
                    mbar_expect(X_FULL + 8 * xs, 2 * XT);
                    tma2d(base + OFF_X + (2 * xs) * XT, &tm_xh, k, n0, X_FULL + 8 * xs);
                    tma2d(base + OFF_X + (2 * xs + 1) * XT, &tm_xl, k, n0, X_FULL + 8 * xs);
                    if constexpr (!QUANT) {
                        const int as = s % A_STAGES;
                        if (s >= A_STAGES)
                            mvtc::wait_or_flag(A_EMPTY + 8 * as, ((s / A_STAGES) - 1) & 1, PCU_DEVERR_EMPTY_WAIT);
                        mbar_expect(A_FULL + 8 * as, TILE);
                        tma2d(base + OFF_A + (2 * as) * TILE, &tm_w, k, m0, A_FULL + 8 * as);
                    }
                }
            }
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA
        if (lane == 0) {
            #pragma unroll 1
            for (int t = blockIdx.x, it = 0; t < total; t += gridDim.x, ++it) {
            // accumulator it & 1; before reusing it, the epilogue must have
            // read out the tile two before this one
            const int buf = it & 1;
            const uint32_t acc = tmem + (uint32_t)(buf * BNT);
            if (it >= 2) {
                mvtc::wait_or_flag(ACC_EMPTY + 8 * buf, ((it >> 1) - 1) & 1, PCU_DEVERR_EMPTY_WAIT);
                tc_after();
            }
            #pragma unroll 1
            for (int s0 = 0; s0 < nks; ++s0) {
                const int s = it * nks + s0;                // step count across tiles
                const int as = s % A_STAGES, xs = s % L::XS;
                mvtc::wait_or_flag(A_FULL + 8 * as, (s / A_STAGES) & 1, PCU_DEVERR_FULL_WAIT);
                mvtc::wait_or_flag(X_FULL + 8 * xs, (s / L::XS) & 1, PCU_DEVERR_FULL_WAIT);
                tc_after();
                const uint32_t ah = base + OFF_A + (2 * as) * TILE, al = ah + TILE;
                const uint32_t xh = base + OFF_X + (2 * xs) * XT, xl = xh + XT;
                #pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    const uint32_t o = 32 * k;        // 16 f16 of a 128-byte swizzled row
                    umma(acc, sdesc(ah + o), sdesc(xh + o), (s0 | k) != 0, ID);
                    umma(acc, sdesc(ah + o), sdesc(xl + o), 1, ID);
                    if constexpr (QUANT) umma(acc, sdesc(al + o), sdesc(xh + o), 1, ID);
                }
                umma_commit(A_EMPTY + 8 * as);
                umma_commit(X_EMPTY + 8 * xs);
            }
            umma_commit(D_FULL + 8 * buf);
            }
        }
    } else if (warp < 2 + DQW) {
        // ----------------------------------------------------------- dequant
        if constexpr (QUANT) {
            const int r = threadIdx.x - 64;                 // weight row within the tile
            #pragma unroll 1
            for (int t = blockIdx.x, it = 0; t < total; t += gridDim.x, ++it) {
            const int m0 = (t % n_mt) * BM;
            const float rsc = (m0 + r < out_n) ? __ldg(rowsc + m0 + r) : 1.f;
            #pragma unroll 1
            for (int kl0 = 0; kl0 < nkb; ++kl0) {
                const int kb = kb0 + kl0, kl = it * nkb + kl0;
                const int rs = kl % RAW_STAGES;
                mvtc::wait_or_flag(RAW_FULL + 8 * rs, (kl / RAW_STAGES) & 1, PCU_DEVERR_FULL_WAIT);
                const uint32_t rw = base + L::OFF_RAW + rs * BM * Raw<TYPE>::B + r * Raw<TYPE>::B;
                #pragma unroll 1
                for (int ks = 0; ks < KB / BK; ++ks) {
                    const int s = kl * (KB / BK) + ks, as = s % A_STAGES;
                    if (s >= A_STAGES)
                        mvtc::wait_or_flag(A_EMPTY + 8 * as, ((s / A_STAGES) - 1) & 1, PCU_DEVERR_EMPTY_WAIT);
                    // hi / lo tiles, row r: 8 chunks of 8 f16, chunk c at (c ^ (r & 7)).
                    const uint32_t ah = base + OFF_A + (2 * as) * TILE + r * 128, al = ah + TILE;
                    auto put = [&](const float* w, int c) {
                        uint4 hv4, lv4;
                        split2(w[0], w[1], hv4.x, lv4.x);
                        split2(w[2], w[3], hv4.y, lv4.y);
                        split2(w[4], w[5], hv4.z, lv4.z);
                        split2(w[6], w[7], hv4.w, lv4.w);
                        const uint32_t off = (uint32_t)((c ^ (r & 7)) << 4);
                        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};"
                                     ::"r"(ah + off), "r"(hv4.x), "r"(hv4.y), "r"(hv4.z), "r"(hv4.w) : "memory");
                        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};"
                                     ::"r"(al + off), "r"(lv4.x), "r"(lv4.y), "r"(lv4.z), "r"(lv4.w) : "memory");
                    };
                    float w[64];                              // the K-step's 64 weights of row r, scaled
                    dequant_kstep<TYPE>(rw, kb, ks, rsc, w);
                    #pragma unroll
                    for (int c = 0; c < 8; ++c) put(w + 8 * c, c);
                    // each thread's tile writes are made visible to the tensor
                    // core (async proxy); then one arrival per warp
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mvtc::mbar_arrive_a(A_FULL + 8 * as);
                }
                __syncwarp();
                if (lane == 0) mvtc::mbar_arrive_a(RAW_EMPTY + 8 * rs);
            }
            }
        }
    } else {
        // ---------------------------------------------------------- epilogue
        const int q = warp & 3;                             // TMEM lanes 32q .. 32q + 31
        // y, or this K slice's partial outputs [n_tok][out_n]
        float* dst = part ? part + (size_t)blockIdx.z * n_tok * out_n : y;
        #pragma unroll 1
        for (int t = blockIdx.x, it = 0; t < total; t += gridDim.x, ++it) {
            const int m0 = (t % n_mt) * BM, n0 = (t / n_mt) * BNT, buf = it & 1;
            const int m = m0 + 32 * q + lane;
            mvtc::wait_or_flag(D_FULL + 8 * buf, (it >> 1) & 1, PCU_DEVERR_MMA_WAIT);
            tc_after();
            const float rinv = (QUANT && m < out_n) ? 1.f / __ldg(rowsc + m) : 1.f;
            #pragma unroll 1
            for (int c = 0; c < BNT / 32; ++c) {
                float v[32];
                tmem_ld32x(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BNT + 32 * c), v);
                // the chunk's 32 token scales: one load per lane, shared by shuffles
                const int nl = n0 + 32 * c + lane;
                const float xs = nl < n_tok ? __ldg(xinv + nl) : 0.f;
                float* d = dst + (size_t)(n0 + 32 * c) * out_n + m;
                // warp-uniform test: all 32 rows and all 32 tokens in range
                if (m0 + 32 * q + 32 <= out_n && n0 + 32 * c + 32 <= n_tok) {
                    #pragma unroll
                    for (int j = 0; j < 32; ++j)
                        d[(size_t)j * out_n] = v[j] * rinv * __shfl_sync(0xffffffffu, xs, j);
                } else {
                    #pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float sj = __shfl_sync(0xffffffffu, xs, j);
                        if (m < out_n && n0 + 32 * c + j < n_tok) d[(size_t)j * out_n] = v[j] * rinv * sj;
                    }
                }
            }
            // this warp has read its lanes of the accumulator out: the MMA
            // may reuse it for the tile after next
            tc_before();
            __syncwarp();
            if (lane == 0) mvtc::mbar_arrive_a(ACC_EMPTY + 8 * buf);
        }
    }
    tc_before();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// Sum of the split-K slices' partial outputs, in slice order:
// y[i] = part[0][i] + part[1][i] + ... (i over n_tok * out_n).
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int ks, size_t total, float* __restrict__ y) {
    griddep_launch_dependents();
    griddep_wait();
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        float a = part[i];
        for (int z = 1; z < ks; ++z) a += part[(size_t)z * total + i];
        y[i] = a;
    }
}

// ---------------------------------------------------------------- host side

// Launch with programmatic stream serialization (the kernels above wait
// with griddepcontrol.wait before they read their inputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess && fn)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return encode;
}

// f16 matrix [rows][cols], 64 x box_rows boxes, 128-byte swizzle.
inline bool map_f16(CUtensorMap* m, const void* p, int cols, int rows, int box_rows) {
    auto enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Raw weight rows [out_n][row_bytes / 8] 64-bit words, box = one K-block x BM rows.
inline bool map_raw(CUtensorMap* m, const void* W, size_t row_bytes, int out_n, int box_bytes) {
    auto enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)out_n};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 8), (cuuint32_t)BM};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(W), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// K slices: when the output tiles do not fill the 148 SMs (a decode batch:
// one token tile), each tile's K-blocks are split over up to 16 CTAs.
constexpr int kSms = 148;
inline int split_k(int out_n, int in_n, int n_tok) {
    const int bn = bn_for(n_tok);
    const long long tiles = (long long)((out_n + BM - 1) / BM) * ((n_tok + bn - 1) / bn);
    const int nkb = in_n / KB;
    if (tiles >= kSms || nkb < 2) return 1;
    int ks = (int)(kSms / tiles);
    if (ks > 16) ks = 16;
    if (ks > nkb) ks = nkb;
    return ks < 1 ? 1 : ks;
}

// Workspace: x hi, x lo [n_tok][in_n] f16, xinv [n_tok], rowsc [out_n],
// and the split-K partials [ks][n_tok][out_n] when ks > 1.
inline size_t workspace_bytes(int out_n, int in_n, int n_tok) {
    const int ks = split_k(out_n, in_n, n_tok);
    return 2 * align256((size_t)n_tok * in_n * 2) + align256((size_t)n_tok * 4) + align256((size_t)out_n * 4) +
           (ks > 1 ? align256((size_t)ks * n_tok * out_n * 4) : 0);
}

// Rows that are 16-byte multiples (TMA) and whole 256-element K-blocks.
inline bool supported(const void* W, size_t row_bytes, int in_n) {
    return reinterpret_cast<uintptr_t>(W) % 16 == 0 && row_bytes % 16 == 0 && in_n % KB == 0;
}

template <int TYPE, int BNT>
inline cudaError_t launch_bn(const uint8_t* W, size_t row_bytes, int out_n, int in_n, int n_tok, const float* x,
                          float* y, void* ws, cudaStream_t st, const float* rowsc_pre = nullptr) {
    uint8_t* p = static_cast<uint8_t*>(ws);
    const size_t plane = align256((size_t)n_tok * in_n * 2);
    __half* xh = reinterpret_cast<__half*>(p);
    __half* xl = reinterpret_cast<__half*>(p + plane);
    float* xinv = reinterpret_cast<float*>(p + 2 * plane);
    float* rowsc = reinterpret_cast<float*>(p + 2 * plane + align256((size_t)n_tok * 4));
    const int ks = split_k(out_n, in_n, n_tok);
    float* part = ks > 1 ? reinterpret_cast<float*>(p + 2 * plane + align256((size_t)n_tok * 4) +
                                                    align256((size_t)out_n * 4))
                         : nullptr;
    if (launch_pdl(xsplit_kernel, dim3(n_tok), dim3(256), 0, st, x, in_n, xh, xl, xinv) != cudaSuccess)
        return cudaGetLastError();
    if constexpr (TYPE != F_F16) {
        // the row scales of constant weights may come precomputed
        if (rowsc_pre) rowsc = const_cast<float*>(rowsc_pre);
        else rowscale_kernel<TYPE><<<(out_n + 7) / 8, 256, 0, st>>>(W, row_bytes, out_n, in_n, rowsc);
    }
    alignas(64) CUtensorMap tw, th, tl;
    const bool ok = (TYPE == F_F16 ? map_f16(&tw, W, in_n, out_n, BM) : map_raw(&tw, W, row_bytes, out_n, Raw<TYPE>::B)) &&
                    map_f16(&th, xh, in_n, n_tok, BNT) && map_f16(&tl, xl, in_n, n_tok, BNT);
    if (!ok) return cudaErrorInvalidValue;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr[dev]) {
        cudaError_t e =
            cudaFuncSetAttribute(matmul_tc_kernel<TYPE, BNT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Lay<TYPE, BNT>::BYTES);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    // Persistent: at most one CTA per SM, each walking its output tiles
    // (one tile per CTA when K is split).
    const int total = ((out_n + BM - 1) / BM) * ((n_tok + BNT - 1) / BNT);
    const dim3 grid((unsigned)(ks > 1 || total < kSms ? total : kSms), 1u, (unsigned)ks);
    cudaError_t e = launch_pdl(matmul_tc_kernel<TYPE, BNT>, grid, dim3(Cfg<BNT>::THREADS), (size_t)Lay<TYPE, BNT>::BYTES,
                               st, tw, th, tl, out_n, in_n, n_tok, (const float*)xinv, (const float*)rowsc, y, part);
    if (e != cudaSuccess) return e;
    if (ks > 1) {
        const size_t total = (size_t)n_tok * out_n;
        const unsigned blocks = (unsigned)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
        e = launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, st, (const float*)part, ks, total, y);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

template <int TYPE>
inline cudaError_t launch(const uint8_t* W, size_t row_bytes, int out_n, int in_n, int n_tok, const float* x,
                          float* y, void* ws, cudaStream_t st, const float* rowsc_pre = nullptr) {
    switch (bn_for(n_tok)) {
        case 32: return launch_bn<TYPE, 32>(W, row_bytes, out_n, in_n, n_tok, x, y, ws, st, rowsc_pre);
        case 64: return launch_bn<TYPE, 64>(W, row_bytes, out_n, in_n, n_tok, x, y, ws, st, rowsc_pre);
        default: return launch_bn<TYPE, 128>(W, row_bytes, out_n, in_n, n_tok, x, y, ws, st, rowsc_pre);
    }
}

// The per-row power-of-two weight scales the GEMM uses, computed once for
// weights that do not change (rowsc [out_n]).
template <int TYPE>
inline cudaError_t rowscale(const uint8_t* W, size_t row_bytes, int out_n, int in_n, float* rowsc, cudaStream_t st) {
    if constexpr (TYPE != F_F16) rowscale_kernel<TYPE><<<(out_n + 7) / 8, 256, 0, st>>>(W, row_bytes, out_n, in_n, rowsc);
    return cudaGetLastError();
}

}  // namespace mmtc
