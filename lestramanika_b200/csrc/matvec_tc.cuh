// matvec_tc.cuh - y = W x for raw GGML weight blocks, streamed through
// shared memory by TMA tensor copies and multiplied on the tensor cores.
//
// The reference dequantizes every weight to float and takes float dot
// products (src/pickle_fast.c:122-1419, dispatched by
// pickle_fast_matmul_dispatch :1423-1474). A GPU doing the same on the CUDA
// cores spends ~17 instructions per weight and cannot keep HBM busy. Here:
//
//   * one persistent CTA per SM takes 16-row tiles of W (tile i, i + grid,
//     ...). One producer lane streams each tile through a ring of
//     shared-memory stages with 2-D TMA tensor copies (a 16-row box of
//     about a kilobyte per row, one copy per stage, no multicast);
//   * x is converted once per CTA, by all its threads, into resident f16
//     "hi + lo" planes: x * 2^s = hi + lo with hi = f16(x * 2^s), lo =
//     f16(x * 2^s - hi) - 22 significant bits, the power of two s chosen
//     per group of 64 elements so the group's largest |x| sits just below
//     2^15 (every accumulator column sees one group between rescales);
//   * CW consumer warps share a tile: warp w takes the tile's blocks b with
//     b % CW == w, turns the quants into exact small f16 integers with a
//     couple of bit operations and runs mma.sync m16n8k16 (f16 in, f32
//     accumulate; A = the 16 rows x 16 k, B = x hi / lo). Their partial sums
//     are added in a fixed order at the end of the tile.
//
// B is block-diagonal: lane quad t owns the k slots {2t, 2t+1, 2t+8, 2t+9}
// of every MMA and only columns 2t (hi) and 2t+1 (lo) of B are non-zero
// in those slots, so accumulator columns 2t / 2t+1 hold the dot product of
// lane quad t's own elements. Each lane therefore applies the scales of
// the block (or sub-block) its own elements come from, and the four
// quads' partial sums are added at the end. Products of an f16 integer and
// an 11-bit f16 are exact in f32, so the result differs from the
// reference's float arithmetic by rounding only.
//
// Every mbarrier wait is bounded (kWaitLimitNs); a timeout records an
// error in g_mv_err and the kernel carries on (results are then garbage,
// but every access stays in bounds and the CTA drains its copies before
// exiting).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "pcu_common.cuh"

namespace mvtc {

constexpr int RT = 16;          // rows per tile (one MMA M)
constexpr int NBOX = 2;         // TMA boxes per stage
constexpr int MAX_STAGES = 4;
constexpr int NRED = MAX_STAGES + 1;   // tile partial-sum buffers (a warp runs at most MAX_STAGES tiles ahead)

enum : int { F_F16 = 1, F_Q4_0 = 2, F_Q8_0 = 8, F_Q4_K = 12, F_Q6_K = 14 };

// Per format: BE elements / BB bytes per block; SEGB blocks per TMA box
// (a stage is NBOX boxes side by side in W, one after the other in shared
// memory); PITCH shared-memory bytes per row of a box (the box width: its
// blocks plus a few bytes of the next ones, for bank spread);
// PERM: x stored as elements (0, 2, 1, 3) of every group of 4 (the order
// the nibble / byte unpacking produces); XSUM: per-32 sums of x kept;
// LOPAD: extra halves between a vector's hi and lo planes; ZOFF: bank
// offset (bytes mod 128) of the zero area the lanes with an all-zero B
// fragment read instead of x.
template <int TYPE> struct Fmt;
// (Every box starts on a 16-byte boundary of its row: SEGB * BB % 16 == 0.)
template <> struct Fmt<F_F16> {
    static constexpr int BE = 64, BB = 128, SEGB = 8, PITCH = 1056, PERM = 0, XSUM = 0, LOPAD = 16, ZOFF = 64;
};
template <> struct Fmt<F_Q4_K> {
    static constexpr int BE = 256, BB = 144, SEGB = 8, PITCH = 1168, PERM = 1, XSUM = 1, LOPAD = 8, ZOFF = 8;
};
template <> struct Fmt<F_Q8_0> {
    static constexpr int BE = 32, BB = 34, SEGB = 32, PITCH = 1168, PERM = 1, XSUM = 0, LOPAD = 16, ZOFF = 64;
};
template <> struct Fmt<F_Q6_K> {
    static constexpr int BE = 256, BB = 210, SEGB = 8, PITCH = 1696, PERM = 1, XSUM = 0, LOPAD = 8, ZOFF = 8;
};
template <> struct Fmt<F_Q4_0> {
    static constexpr int BE = 32, BB = 18, SEGB = 64, PITCH = 1168, PERM = 1, XSUM = 0, LOPAD = 16, ZOFF = 64;
};

// Consumer warps: 16 (four per SM sub-partition) while the registers of a
// thread allow it, 8 for the widest accumulator sets (Q6_K keeps four per
// vector and row pair).
__host__ __device__ constexpr int consumer_warps(int type, int nv) { return nv <= (type == F_Q6_K ? 2 : 4) ? 16 : 8; }
template <int TYPE, int NV> struct Warps {
    static constexpr int CW = consumer_warps(TYPE, NV);
    static constexpr int THREADS = 32 * (CW + 1);
};

// Shared-memory layout; the x planes depend on in_n.
struct Smem {
    int stages, stage, plane, lo, vstride, off_x, off_zero, off_xsum, off_xinv, off_red, off_bar, bytes;
};
constexpr int kSmemLimit = 232448;
template <int TYPE>
__host__ __device__ inline Smem smem_layout_n(int in_n, int nv, int cw, int stages) {
    using F = Fmt<TYPE>;
    Smem s;
    s.stages = stages;
    s.stage = NBOX * RT * F::PITCH;
    s.plane = ((in_n + in_n / 4) + 63) & ~63;          // halves, 8 bytes of pad per 16 elements
    s.lo = s.plane + F::LOPAD;
    s.vstride = (2 * s.plane + F::LOPAD + 63) & ~63;
    s.off_x = stages * s.stage;
    s.off_zero = s.off_x + nv * s.vstride * 2 + F::ZOFF;   // 1 KB of zeros
    s.off_xsum = s.off_zero - F::ZOFF + 1024 + 128;
    s.off_xinv = s.off_xsum + (F::XSUM ? nv * (in_n / 32) * 4 : 0);   // [nv][in_n / 64] 2^-s
    s.off_red = (s.off_xinv + nv * (in_n / 64) * 4 + 2 * 4 + 15) & ~15;   // + two multipliers
    s.off_bar = s.off_red + NRED * cw * RT * nv * 4 + 16 * 4;           // + NRED arrival counters
    s.bytes = s.off_bar + 2 * MAX_STAGES * 8;
    return s;
}
// The deepest ring (up to MAX_STAGES) that fits; .bytes > kSmemLimit when
// even two stages do not.
template <int TYPE>
__host__ __device__ inline Smem smem_layout(int in_n, int nv, int cw) {
    Smem s = smem_layout_n<TYPE>(in_n, nv, cw, MAX_STAGES);
    for (int st = MAX_STAGES - 1; st >= 2 && s.bytes > kSmemLimit; --st) s = smem_layout_n<TYPE>(in_n, nv, cw, st);
    return s;
}

// Device error word of the tensor-core matvec (PCU_DEVERR_* codes).
static __device__ int g_mv_err;

// Halves offset of element e (a multiple of 4) within a plane.
PCU_DEV int xa(int e) { return e + 4 * (e >> 4); }

// D += A B, m16n8k16, f16 inputs, f32 accumulate.
PCU_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

// D = A B (accumulator starts at zero).
PCU_DEV void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y), "f"(0.f));
}

// Shared-memory loads by 32-bit shared address (volatile: they stay after
// the mbarrier wait that makes the data valid).
PCU_DEV uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
PCU_DEV uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
PCU_DEV float2 ldsf2(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
PCU_DEV uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
PCU_DEV uint32_t ldsu8(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
PCU_DEV uint32_t ldsu16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
// 16 bytes starting M bytes past the 16-byte aligned shared address a.
template <int M>
PCU_DEV void lds16_at(uint32_t a, uint32_t (&o)[4]) {
    const uint4 p = lds128(a);
    if constexpr (M == 0) {
        o[0] = p.x; o[1] = p.y; o[2] = p.z; o[3] = p.w;
    } else {
        const uint4 q = lds128(a + 16);
        const uint32_t w[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
        #pragma unroll
        for (int k = 0; k < 4; ++k)
            o[k] = (M % 4 == 0) ? w[M / 4 + k] : __funnelshift_r(w[M / 4 + k], w[M / 4 + k + 1], 8 * (M % 4));
    }
}

// Four bytes at a shared address that is 2 (mod 4): two aligned words.
PCU_DEV uint32_t lds32_odd2(uint32_t a) { return __funnelshift_r(lds32(a - 2), lds32(a + 2), 16); }
PCU_DEV float ldsf(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}

// mbarrier operations by 32-bit shared address.
PCU_DEV void mbar_arrive_a(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

PCU_DEV uint32_t __hsub2_u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Byte `which` (0..3) of w as a float, exactly (0x4B000000 | b is 2^23 + b).
PCU_DEV float bytef(uint32_t w, int which) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440 | which)) - 8388608.0f;
}

// Bytes `which` of a and of b as a float pair, exactly.
PCU_DEV float2 bytef2(uint32_t a, uint32_t b, int which) {
    const float2 m = make_float2(__uint_as_float(__byte_perm(a, 0x4B000000u, 0x7440 | which)),
                                 __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7440 | which)));
    return __fadd2_rn(m, make_float2(-8388608.0f, -8388608.0f));
}

PCU_DEV float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
PCU_DEV float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

// try_wait with a suspend-time hint: a waiting warp sleeps until the
// phase completes (or the hint runs out) instead of spinning.
PCU_DEV bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}

PCU_DEV void wait_or_flag(uint32_t bar, uint32_t parity, int code) {
    if (mbar_try_wait_sleep(bar, parity)) return;
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait_sleep(bar, parity))
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            record_error(&g_mv_err, code);
            return;
        }
}
PCU_DEV void wait_or_flag(uint64_t* bar, uint32_t parity, int code) { wait_or_flag(smem_u32(bar), parity, code); }

PCU_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// All threads: x [nv][in_n] into resident hi / lo planes, per-32 sums and
// per-64 scales 2^-s; one pass, 16 lanes per group of 64 elements.
template <int TYPE, int NV, int THREADS>
PCU_DEV void convert_x(const float* __restrict__ x, int in_n, uint8_t* smem, const Smem& L) {
    using F = Fmt<TYPE>;
    const int tid = threadIdx.x, lane = tid & 31;
    __half* xb = reinterpret_cast<__half*>(smem + L.off_x);
    float* xs = reinterpret_cast<float*>(smem + L.off_xsum);
    float* xi = reinterpret_cast<float*>(smem + L.off_xinv);
    const int n64 = in_n / 64;
    #pragma unroll 1
    for (int v = 0; v < NV; ++v) {
        const float* xv = x + (size_t)v * in_n;
        __half* hp = xb + v * L.vstride;
        // Trip count uniform per warp (whole warps take part in the shuffles).
        #pragma unroll 1
        for (int i0 = 4 * (tid - lane); i0 < in_n; i0 += 4 * THREADS) {
            const int i = i0 + 4 * lane;
            const bool in = i < in_n;
            const float4 q = in ? __ldg(reinterpret_cast<const float4*>(xv + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            float m = fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w)));
            #pragma unroll
            for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            int sft = 14 - ((int)((__float_as_uint(m) >> 23) & 0xFF) - 127);
            sft = max(-126, min(126, sft));
            const float sc = __uint_as_float((uint32_t)(127 + sft) << 23);
            const float a[4] = {q.x * sc, q.y * sc, q.z * sc, q.w * sc};
            __half h[4], l[4];
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
                h[k] = __float2half_rn(a[k]);
                l[k] = __float2half_rn(a[k] - __half2float(h[k]));
            }
            const int p1 = F::PERM ? 2 : 1, p2 = F::PERM ? 1 : 2;
            uint2 hv, lv;
            hv.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[p1]) << 16);
            hv.y = (uint32_t)__half_as_ushort(h[p2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
            lv.x = (uint32_t)__half_as_ushort(l[0]) | ((uint32_t)__half_as_ushort(l[p1]) << 16);
            lv.y = (uint32_t)__half_as_ushort(l[p2]) | ((uint32_t)__half_as_ushort(l[3]) << 16);
            float t = (q.x + q.y) + (q.z + q.w);
            t += __shfl_xor_sync(0xffffffffu, t, 1);
            t += __shfl_xor_sync(0xffffffffu, t, 2);
            t += __shfl_xor_sync(0xffffffffu, t, 4);
            if (in) {
                *reinterpret_cast<uint2*>(hp + xa(i)) = hv;
                *reinterpret_cast<uint2*>(hp + L.lo + xa(i)) = lv;
                if constexpr (F::XSUM != 0)
                    if ((lane & 7) == 0) xs[v * (in_n / 32) + i / 32] = t;
                if ((lane & 15) == 0) xi[v * n64 + i / 64] = __uint_as_float((uint32_t)(127 - sft) << 23);
            }
        }
    }
    // Multipliers read back at run time, so that the nibble shifts stay
    // integer multiplies on the FMA pipe instead of becoming shifts on the
    // busier ALU pipe.
    if (tid == 0) {
        reinterpret_cast<uint32_t*>(xi + NV * n64)[0] = 16u;
        reinterpret_cast<uint32_t*>(xi + NV * n64)[1] = 1u << 24;
    }
    for (int i = tid; i < 256; i += THREADS) reinterpret_cast<uint32_t*>(smem + L.off_zero)[i] = 0u;
    if (tid < NRED) reinterpret_cast<int*>(smem + L.off_bar)[-16 + tid] = 0;
}

template <int TYPE, int NV>
__global__ void __launch_bounds__(Warps<TYPE, NV>::THREADS, 1)
    matvec_tc_kernel(const __grid_constant__ CUtensorMap tm, int out_n, int in_n, const float* __restrict__ x,
                     float* __restrict__ y, int w_early) {
    using F = Fmt<TYPE>;
    constexpr int CW = Warps<TYPE, NV>::CW, THREADS = Warps<TYPE, NV>::THREADS;
    extern __shared__ __align__(128) uint8_t smem[];
    const Smem L = smem_layout<TYPE>(in_n, NV, CW);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    const int STAGES = L.stages;
    uint64_t* b_full = bars;                 // [STAGES] TMA bytes landed
    uint64_t* b_empty = bars + MAX_STAGES;   // [STAGES] CW consumer warps done
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = in_n / F::BE;
    constexpr int SB = NBOX * F::SEGB;                            // blocks per stage
    const int spt = (nb + SB - 1) / SB;                           // stages per tile
    const int n_tiles = (out_n + RT - 1) / RT;
    const int my_tiles = n_tiles > (int)blockIdx.x ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_st = my_tiles * spt;
    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], CW);
        }
        mbar_fence_init();
    }
    __syncthreads();

    // Stage s of this CTA: blocks [j * SB, +SB) of tile (the CTA's k-th),
    // into ring slot s % STAGES; slot, phase, j and k advance incrementally.
    auto issue = [&](int slot, int k, int j) {
        const int tile = (int)blockIdx.x + k * (int)gridDim.x;
        const int nbox = min(NBOX, (nb - j * SB + F::SEGB - 1) / F::SEGB);
        mbar_arrive_expect_tx(&b_full[slot], (uint32_t)(nbox * RT * F::PITCH));
        for (int i = 0; i < nbox; ++i)
            tma_load_2d(smem + slot * L.stage + i * RT * F::PITCH, &tm, (j * SB + i * F::SEGB) * F::BB / 8,
                        tile * RT, &b_full[slot]);
    };
    int p_slot = 0, p_k = 0, p_j = 0;              // producer position
    auto p_next = [&]() {
        if (++p_j == spt) { p_j = 0; ++p_k; }
        if (++p_slot == STAGES) p_slot = 0;
    };
    // Launched with programmatic stream serialization: let the next kernel
    // be scheduled now, and read nothing the previous kernel may write
    // before it has completed. W is such memory unless the caller says it
    // is constant (w_early): then the first stages of W are already on
    // their way while the previous kernel finishes.
    griddep_launch_dependents();
    if (!w_early) griddep_wait();
    if (warp == CW && lane == 0)
        for (int s = 0; s < min(STAGES, n_st); ++s) {
            issue(p_slot, p_k, p_j);
            p_next();
        }
    if (w_early) griddep_wait();
    convert_x<TYPE, NV, THREADS>(x, in_n, smem, L);
    __syncthreads();

    if (warp == CW) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            uint32_t e_phase = 0;                  // phase of b_empty[p_slot] to wait for
            #pragma unroll 1
            for (int s = STAGES; s < n_st; ++s) {
                wait_or_flag(&b_empty[p_slot], e_phase, PCU_DEVERR_EMPTY_WAIT);
                issue(p_slot, p_k, p_j);
                if (p_slot == STAGES - 1) e_phase ^= 1;
                p_next();
            }
            // Every copy must have landed before the CTA may exit.
            for (int s = max(0, n_st - STAGES); s < n_st; ++s)
                wait_or_flag(&b_full[s % STAGES], (s / STAGES) & 1, PCU_DEVERR_DRAIN_WAIT);
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    // Lane (g, t) carries B column g in quad t's k slots: x hi (g = 2t) or
    // lo (g = 2t + 1) of quad t's elements, zeros elsewhere. Lanes with a
    // zero fragment read the zero area at the same relative offsets.
    const bool act = (g >> 1) == t;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t xpl = act ? sbase + L.off_x + ((g & 1) ? 2 * L.lo : 0) : sbase + L.off_zero;   // bytes
    const int xact = act ? 2 : 0;                    // 0: ignore the element offset of the block
    const uint32_t vstep = act ? 2 * L.vstride : 0;
    const uint32_t xsum = sbase + L.off_xsum, xinv = sbase + L.off_xinv;
    const uint32_t full0 = smem_u32(b_full), empty0 = smem_u32(b_empty);
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    const int n64 = in_n / 64;
    const uint32_t k16 = reinterpret_cast<const uint32_t*>(smem + L.off_xinv)[NV * n64];
    const uint32_t k24 = reinterpret_cast<const uint32_t*>(smem + L.off_xinv)[NV * n64 + 1];

    int slot = 0;
    uint32_t f_phase = 0;
    #pragma unroll 1
    for (int k = 0; k < my_tiles; ++k) {
        float acc[NV][2];
        #pragma unroll
        for (int v = 0; v < NV; ++v) acc[v][0] = acc[v][1] = 0.f;
        #pragma unroll 1
        for (int j = 0; j < spt; ++j) {
            wait_or_flag(full0 + 8 * slot, f_phase, PCU_DEVERR_FULL_WAIT);
            const int nblk = min(SB, nb - j * SB);
            #pragma unroll 1
            for (int bb = warp; bb < nblk; bb += CW) {
                const int e = (j * SB + bb) * F::BE;               // first element of the block
                const int lb = bb % F::SEGB;                      // block within its box
                // This lane's row g of the block (row g + 8 is 8 * PITCH further).
                const uint32_t rg = sbase + slot * L.stage + (bb / F::SEGB) * (RT * F::PITCH) + g * F::PITCH +
                                    lb * F::BB;
                if constexpr (TYPE == F_F16) {
                    // Block = 64 halves of a row; MMA i takes halves
                    // 16i + 4t .. +3 of rows g and g + 8 as lane (g, t)'s k slots.
                    const uint32_t ra = rg + 8 * t;
                    const uint32_t xb = xpl + xact * xa(e) + 8 * t;
                    float D[NV][4];
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint2 a = lds64(ra + 32 * i), a8 = lds64(ra + 8 * F::PITCH + 32 * i);
                        #pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const uint2 b = lds64(xb + v * vstep + 40 * i);
                            if (i == 0) mma16816_z(D[v], a.x, a8.x, a.y, a8.y, b);
                            else mma16816(D[v], a.x, a8.x, a.y, a8.y, b);
                        }
                    }
                    #pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float inv = ldsf(xinv + 4 * (v * n64 + e / 64));
                        float2 a2 = make_float2(acc[v][0], acc[v][1]);
                        a2 = __ffma2_rn(make_float2(inv, inv),
                                        __fadd2_rn(make_float2(D[v][0], D[v][2]), make_float2(D[v][1], D[v][3])), a2);
                        acc[v][0] = a2.x;
                        acc[v][1] = a2.y;
                    }
                } else if constexpr (TYPE == F_Q8_0 || TYPE == F_Q4_0) {
                    // 32-element blocks: d (f16) then the quants. Lane quad t
                    // takes elements 4t .. 4t+3 (MMA 0) and 16+4t .. 16+4t+3
                    // (MMA 1): for Q8_0 quant bytes 4t and 16+4t, for Q4_0 the
                    // low and high nibbles of quant bytes 4t .. 4t+3. The quants
                    // start 2 bytes into the block, so they are 4-byte aligned
                    // in odd blocks only; the parity of the block within its box
                    // is that of the warp (blocks go to warps modulo 16).
                    const uint32_t rq = rg + 2 + 4 * t, rq8 = rq + 8 * F::PITCH;
                    const bool odd = (lb & 1) != 0;
                    uint32_t a[2][2];                               // [row g / g + 8][mma]
                    if constexpr (TYPE == F_Q8_0) {
                        a[0][0] = odd ? lds32(rq) : lds32_odd2(rq);
                        a[0][1] = odd ? lds32(rq + 16) : lds32_odd2(rq + 16);
                        a[1][0] = odd ? lds32(rq8) : lds32_odd2(rq8);
                        a[1][1] = odd ? lds32(rq8 + 16) : lds32_odd2(rq8 + 16);
                    } else {
                        a[0][0] = a[0][1] = odd ? lds32(rq) : lds32_odd2(rq);
                        a[1][0] = a[1][1] = odd ? lds32(rq8) : lds32_odd2(rq8);
                    }
                    const uint32_t xb = xpl + xact * xa(e) + 8 * t;
                    float D[NV][4];
                    #pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        uint32_t p02[2], p13[2];
                        #pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            const uint32_t w = a[r][m];
                            if constexpr (TYPE == F_Q8_0) {
                                // signed bytes: (b + 128) under the 1024 magic, less 1152
                                constexpr uint32_t H = 0x64006400u, C = 0x64806480u;   // 1024, 1152
                                p02[r] = __hsub2_u(((w ^ 0x80808080u) & 0x00FF00FFu) | H, C);
                                p13[r] = __hsub2_u((((w >> 8) ^ 0x00800080u) & 0x00FF00FFu) | H, C);
                            } else {
                                // nibble m of each byte, q - 8: 1024 + q less 1032,
                                // or 64 + q less 72 for the high nibble
                                if (m == 0) {
                                    p02[r] = __hsub2_u((w & 0x000F000Fu) | 0x64006400u, 0x64086408u);
                                    p13[r] = __hsub2_u(((w >> 8) & 0x000F000Fu) | 0x64006400u, 0x64086408u);
                                } else {
                                    p02[r] = __hsub2_u((w & 0x00F000F0u) | 0x54005400u, 0x54805480u);
                                    p13[r] = __hsub2_u(((w >> 8) & 0x00F000F0u) | 0x54005400u, 0x54805480u);
                                }
                            }
                        }
                        #pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const uint2 b = lds64(xb + v * vstep + 40 * m);   // elements +16m: 20 halves
                            if (m == 0) mma16816_z(D[v], p02[0], p02[1], p13[0], p13[1], b);
                            else mma16816(D[v], p02[0], p02[1], p13[0], p13[1], b);
                        }
                    }
                    // d of rows g, g + 8 (2-byte aligned).
                    const float d0 = __half2float(__ushort_as_half((unsigned short)ldsu16(rg)));
                    const float d1 = __half2float(__ushort_as_half((unsigned short)ldsu16(rg + 8 * F::PITCH)));
                    #pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float inv = ldsf(xinv + 4 * (v * n64 + e / 64));
                        acc[v][0] = fmaf(d0 * inv, D[v][0] + D[v][1], acc[v][0]);
                        acc[v][1] = fmaf(d1 * inv, D[v][2] + D[v][3], acc[v][1]);
                    }
                } else if constexpr (TYPE == F_Q6_K) {
                    // 256-element blocks: ql[128], qh[64], int8 scales[16], d
                    // (src/pickle_fast.c:1084-1257). Element 128n + 32u + l
                    // (u = 0..3, l = 0..31) is (low 4 bits from ql[64n + l +
                    // 32 (u & 1)], low nibble for u < 2, high for u >= 2) | ((qh[32n
                    // + l] >> 2u) & 3) << 4, less 32, times scales[8n + l/16 + 2u].
                    // Lane quad t = 2n + h takes l = 16h .. 16h + 15 of half n: 16
                    // bytes of ql at 64n + 16h (u = 0, 2) and 64n + 32 + 16h (u = 1,
                    // 3), 16 of qh at 128 + 32n + 16h; one scale per u. The block
                    // sits 2 lb bytes past a 16-byte boundary (lb = warp % 8 here).
                    const int n = t >> 1, hh = t & 1;
                    const uint32_t ab = rg - 2 * lb;               // 16-byte aligned block start
                    const int oA = 64 * n + 16 * hh, oB = oA + 32, oH = 128 + 32 * n + 16 * hh;
                    uint32_t qa[2][4], qb[2][4], qh[2][4];
                    auto load = [&](auto mc) {
                        constexpr int M = decltype(mc)::value;
                        #pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            const uint32_t rb0 = ab + r * 8 * F::PITCH;
                            lds16_at<M>(rb0 + oA, qa[r]);
                            lds16_at<M>(rb0 + oB, qb[r]);
                            lds16_at<M>(rb0 + oH, qh[r]);
                        }
                    };
                    switch (lb) {
                        case 0: load(std::integral_constant<int, 0>{}); break;
                        case 1: load(std::integral_constant<int, 2>{}); break;
                        case 2: load(std::integral_constant<int, 4>{}); break;
                        case 3: load(std::integral_constant<int, 6>{}); break;
                        case 4: load(std::integral_constant<int, 8>{}); break;
                        case 5: load(std::integral_constant<int, 10>{}); break;
                        case 6: load(std::integral_constant<int, 12>{}); break;
                        default: load(std::integral_constant<int, 14>{}); break;
                    }
                    const uint32_t xb = xpl + xact * xa(e) + 2 * (160 * n + 20 * hh);
                    float D[NV][4][4];                              // [v][u][fragment]
                    constexpr uint32_t H = 0x64006400u, C = 0x64206420u;   // 1024, 1056
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        #pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            uint32_t p02[2], p13[2];
                            #pragma unroll
                            for (int r = 0; r < 2; ++r) {
                                const uint32_t ql = (u & 1) ? qb[r][i] : qa[r][i];
                                const uint32_t lo4 = u < 2 ? ql : ql >> 4;              // nibble at bits 0-3
                                const uint32_t hq = qh[r][i];
                                // qh bits 2u, 2u+1 of bytes 0, 2 to bits 4, 5 (and of
                                // bytes 1, 3 after the >> 8 below).
                                const uint32_t h2 = u == 0 ? hq << 4 : u == 1 ? hq << 2 : u == 2 ? hq : hq >> 2;
                                p02[r] = __hsub2_u(((lo4 & 0x000F000Fu) | H) | (h2 & 0x00300030u), C);
                                p13[r] = __hsub2_u((((lo4 >> 8) & 0x000F000Fu) | H) | ((h2 >> 8) & 0x00300030u), C);
                            }
                            #pragma unroll
                            for (int v = 0; v < NV; ++v) {
                                const uint2 b = lds64(xb + v * vstep + 2 * (40 * u + 4 * i));   // +32u + 4i elements
                                if (i == 0) mma16816_z(D[v][u], p02[0], p02[1], p13[0], p13[1], b);
                                else mma16816(D[v][u], p02[0], p02[1], p13[0], p13[1], b);
                            }
                        }
                    }
                    // d * scale per u for rows g, g + 8.
                    float ds[2][4];
                    #pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const uint32_t rr = rg + r * 8 * F::PITCH;
                        const float d = __half2float(__ushort_as_half((unsigned short)ldsu16(rr + 208)));
                        #pragma unroll
                        for (int u = 0; u < 4; ++u)
                            ds[r][u] = d * (float)(int)(signed char)ldsu8(rr + 192 + 8 * n + hh + 2 * u);
                    }
                    #pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        // u = 0, 1 lie in 64-group 4e/256 + 2n, u = 2, 3 in the next one
                        const float2 iv = ldsf2(xinv + 4 * (v * n64 + e / 64 + 2 * n));
                        #pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            const float s01 = fmaf(ds[r][0], D[v][0][2 * r] + D[v][0][2 * r + 1],
                                                   ds[r][1] * (D[v][1][2 * r] + D[v][1][2 * r + 1]));
                            const float s23 = fmaf(ds[r][2], D[v][2][2 * r] + D[v][2][2 * r + 1],
                                                   ds[r][3] * (D[v][3][2 * r] + D[v][3][2 * r + 1]));
                            acc[v][r] = fmaf(iv.x, s01, fmaf(iv.y, s23, acc[v][r]));
                        }
                    }
                } else if constexpr (TYPE == F_Q4_K) {
                    // Lane quad t takes chunk t (qs bytes 32t .. 32t+31) of the
                    // block: low nibbles = sub-block 2t, high nibbles = 2t + 1.
                    // Quants enter the MMA as 64 + q (exact f16); the 64 * sum(x)
                    // this adds comes off with the sub-block's x sum.
                    const uint32_t rq = rg + 16 + 32 * t;
                    const uint4 qa = lds128(rq), qb = lds128(rq + 16);
                    const uint4 qa8 = lds128(rq + 8 * F::PITCH), qb8 = lds128(rq + 8 * F::PITCH + 16);
                    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    const uint32_t w8[8] = {qa8.x, qa8.y, qa8.z, qa8.w, qb8.x, qb8.y, qb8.z, qb8.w};
                    const uint32_t xb = xpl + xact * xa(e) + 160 * t;   // xa(e + 64t) = xa(e) + 80t halves
                    float D[NV][2][4];
                    constexpr uint32_t M = 0x00F000F0u, H64 = 0x54005400u;   // f16 64.0, ulp 1/16
                    #pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int xo = 4 * i + 4 * (i >> 2);
                        // u = w >> 8; w * 16 and u * 16 put the low nibbles of
                        // bytes (0, 2) and (1, 3) where the high ones of w and u are.
                        const uint32_t u = __umulhi(w[i], k24), u8 = __umulhi(w8[i], k24);
                        const uint32_t l0 = ((w[i] * k16) & M) | H64, l2 = ((u * k16) & M) | H64;
                        const uint32_t l1 = ((w8[i] * k16) & M) | H64, l3 = ((u8 * k16) & M) | H64;
                        #pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const uint2 b = lds64(xb + v * vstep + 2 * xo);
                            if (i == 0) mma16816_z(D[v][0], l0, l1, l2, l3, b);
                            else mma16816(D[v][0], l0, l1, l2, l3, b);
                        }
                        const uint32_t h0 = (w[i] & M) | H64, h2 = (u & M) | H64;
                        const uint32_t h1 = (w8[i] & M) | H64, h3 = (u8 & M) | H64;
                        #pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const uint2 b = lds64(xb + v * vstep + 80 + 2 * xo);
                            if (i == 0) mma16816_z(D[v][1], h0, h1, h2, h3, b);
                            else mma16816(D[v][1], h0, h1, h2, h3, b);
                        }
                    }
                    // Scales and mins of sub-blocks 2t, 2t + 1 of rows g, g + 8
                    // (6-bit, packed in header bytes 4..15:
                    // src/pickle_fast.c:368-383): for t < 2 the low 6 bits of
                    // bytes 2t, 2t+1 (scales) and 4+2t, 5+2t (mins); for t >= 2
                    // the nibbles of bytes 8+.. with the top 2 bits of bytes
                    // 0+.. (scales) and 4+.. (mins) above them.
                    const uint4 hg = lds128(rg), hg8 = lds128(rg + 8 * F::PITCH);
                    const int sh = 16 * (t & 1);
                    const uint32_t MA = t < 2 ? 0x3F3Fu : 0x0F0Fu, MB = t < 2 ? 0u : 0x3030u;
                    const int shm = t < 2 ? sh : sh + 4;
                    auto dec = [&](const uint4& h, uint32_t& sc2, uint32_t& m2) {
                        const uint32_t X = t < 2 ? h.y : h.w, Y = t < 2 ? h.z : h.w;
                        sc2 = ((X >> sh) & MA) | ((h.y >> (sh + 2)) & MB);
                        m2 = ((Y >> shm) & MA) | ((h.z >> (sh + 2)) & MB);
                    };
                    uint32_t sc_g, m_g, sc_g8, m_g8;
                    dec(hg, sc_g, m_g);
                    dec(hg8, sc_g8, m_g8);
                    const float2 d2 = make_float2(h2f_lo(hg.x), h2f_lo(hg8.x));
                    const float2 dm2 = make_float2(h2f_hi(hg.x), h2f_hi(hg8.x));
                    const float2 da = __fmul2_rn(d2, bytef2(sc_g, sc_g8, 0));
                    const float2 db = __fmul2_rn(d2, bytef2(sc_g, sc_g8, 1));
                    const float2 c64 = make_float2(64.f, 64.f);
                    const float2 ca = __ffma2_rn(c64, da, __fmul2_rn(dm2, bytef2(m_g, m_g8, 0)));
                    const float2 cb = __ffma2_rn(c64, db, __fmul2_rn(dm2, bytef2(m_g, m_g8, 1)));
                    const int sub = e / 32 + 2 * t;
                    #pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float2 xs2 = ldsf2(xsum + 4 * (v * (in_n / 32) + sub));
                        const float2 lo = __fadd2_rn(make_float2(D[v][0][0], D[v][0][2]), make_float2(D[v][0][1], D[v][0][3]));
                        const float2 hi = __fadd2_rn(make_float2(D[v][1][0], D[v][1][2]), make_float2(D[v][1][1], D[v][1][3]));
                        float2 a = make_float2(acc[v][0], acc[v][1]);
                        const float inv = ldsf(xinv + 4 * (v * n64 + e / 64 + t));   // quad t's 64 elements
                        a = __ffma2_rn(make_float2(inv, inv), __ffma2_rn(da, lo, __fmul2_rn(db, hi)), a);
                        a = __ffma2_rn(make_float2(-ca.x, -ca.y), make_float2(xs2.x, xs2.x), a);
                        a = __ffma2_rn(make_float2(-cb.x, -cb.y), make_float2(xs2.y, xs2.y), a);
                        acc[v][0] = a.x;
                        acc[v][1] = a.y;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_a(empty0 + 8 * slot);
            if (++slot == STAGES) {
                slot = 0;
                f_phase ^= 1;
            }
        }

        // Tile end: sum the lane quads and post this warp's partials; the
        // last warp to post sums all CW of them in warp order (the result
        // does not depend on which warp that is) and writes y.
        const int rbi = k % NRED;
        float* rb = red + rbi * CW * RT * NV;              // [row * NV + v][warp]
        int* cnt = reinterpret_cast<int*>(smem + L.off_bar) - 16;
        #pragma unroll
        for (int v = 0; v < NV; ++v)
            #pragma unroll
            for (int r = 0; r < 2; ++r) {
                float a = acc[v][r];
                a += __shfl_xor_sync(0xffffffffu, a, 1);
                a += __shfl_xor_sync(0xffffffffu, a, 2);
                if (t == 0) rb[((g + 8 * r) * NV + v) * CW + warp] = a;
            }
        __syncwarp();
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(&cnt[rbi], 1);
            __threadfence_block();
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        __syncwarp();
        if (old == CW - 1) {
            constexpr int NO = RT * NV;                    // outputs of the tile
            constexpr int LPO = NO >= 32 ? 1 : 32 / NO;    // lanes per output
            constexpr int PPL = CW / LPO;                  // partials per lane (a multiple of 4)
            #pragma unroll 1
            for (int o0 = 0; o0 < NO; o0 += 32 / LPO) {
                const int o = o0 + lane / LPO;
                float a = 0.f;
                if (o < NO) {
                    const float4* src = reinterpret_cast<const float4*>(rb + o * CW + (lane % LPO) * PPL);
                    #pragma unroll
                    for (int q = 0; q < PPL / 4; ++q) {
                        const float4 p4 = src[q];
                        a += (p4.x + p4.y) + (p4.z + p4.w);
                    }
                }
                #pragma unroll
                for (int m = LPO / 2; m > 0; m >>= 1) a += __shfl_xor_sync(0xffffffffu, a, m);
                if (lane % LPO == 0 && o < NO) {
                    const int r = o / NV, v = o % NV;
                    const int row = ((int)blockIdx.x + k * (int)gridDim.x) * RT + r;
                    if (row < out_n) y[(size_t)v * out_n + row] = a;
                }
            }
            if (lane == 0) cnt[rbi] = 0;
        }
    }
}

// 2-D tensor map over W as [out_n rows][row_bytes / 8] 64-bit words; box =
// PITCH bytes x 16 rows (rows past out_n and bytes past a row's end are
// filled with zeros).
template <int TYPE>
inline int make_w_map(CUtensorMap* map, const void* W, size_t row_bytes, int out_n) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
            return -1;
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)out_n};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(Fmt<TYPE>::PITCH / 8), (cuuint32_t)RT};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(W), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -1;
}

// True when the tensor-core path takes this call (otherwise the caller
// uses the CUDA-core kernel): 16-byte aligned rows, whole blocks, and x
// of one vector fitting in shared memory next to the ring.
template <int TYPE>
inline bool tc_supported(const void* W, size_t row_bytes, int in_n) {
    if (reinterpret_cast<uintptr_t>(W) % 16 || row_bytes % 16 || in_n % Fmt<TYPE>::BE) return false;
    if (Fmt<TYPE>::XSUM && in_n % 256) return false;
    return smem_layout<TYPE>(in_n, 1, Warps<TYPE, 1>::CW).bytes <= kSmemLimit;
}

// Vectors one pass over W can take: as many (up to 8) as fit in shared
// memory beside a two-stage ring.
template <int TYPE>
inline int fit_nv(int in_n) {
    int nv = 8;
    while (nv > 1 && smem_layout<TYPE>(in_n, nv, consumer_warps(TYPE, nv)).bytes > kSmemLimit) --nv;
    return nv;
}

template <int TYPE, int NV>
inline cudaError_t launch_nv(const CUtensorMap& tm, int out_n, int in_n, const float* x, float* y, cudaStream_t st,
                             bool w_early) {
    const Smem L = smem_layout<TYPE>(in_n, NV, Warps<TYPE, NV>::CW);
    static bool attr_set[64] = {};
    static int sms[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(matvec_tc_kernel<TYPE, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemLimit);
        if (e != cudaSuccess) return e;
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        attr_set[dev] = true;
    }
    const int n_tiles = (out_n + RT - 1) / RT;
    const int grid = n_tiles < sms[dev] ? n_tiles : sms[dev];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(Warps<TYPE, NV>::THREADS);
    cfg.dynamicSmemBytes = (size_t)L.bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, matvec_tc_kernel<TYPE, NV>, tm, out_n, in_n, x, y, (int)w_early);
}

template <int TYPE>
inline cudaError_t launch(const uint8_t* W, size_t row_bytes, int out_n, int in_n, int n_vec, const float* x,
                          float* y, cudaStream_t st, bool w_early = false) {
    alignas(64) CUtensorMap tm;
    if (make_w_map<TYPE>(&tm, W, row_bytes, out_n) != 0) return cudaErrorInvalidValue;
    // Vectors go in passes of at most as many as fit in shared memory, the
    // same number in each pass (8 that fit 7 at a time go as 4 + 4, not
    // 7 + 1): as many passes over W, and narrower passes keep more
    // consumer warps.
    const int fit = fit_nv<TYPE>(in_n);
    const int passes = (n_vec + fit - 1) / fit;
    const int per = (n_vec + passes - 1) / passes;
    for (int v0 = 0; v0 < n_vec;) {
        const int nv = n_vec - v0 < per ? n_vec - v0 : per;
        const float* xv = x + (size_t)v0 * in_n;
        float* yv = y + (size_t)v0 * out_n;
        cudaError_t e = cudaSuccess;
        switch (nv) {
            case 1: e = launch_nv<TYPE, 1>(tm, out_n, in_n, xv, yv, st, w_early); break;
            case 2: e = launch_nv<TYPE, 2>(tm, out_n, in_n, xv, yv, st, w_early); break;
            case 3: e = launch_nv<TYPE, 3>(tm, out_n, in_n, xv, yv, st, w_early); break;
            case 4: e = launch_nv<TYPE, 4>(tm, out_n, in_n, xv, yv, st, w_early); break;
            case 5: e = launch_nv<TYPE, 5>(tm, out_n, in_n, xv, yv, st, w_early); break;
            case 6: e = launch_nv<TYPE, 6>(tm, out_n, in_n, xv, yv, st, w_early); break;
            case 7: e = launch_nv<TYPE, 7>(tm, out_n, in_n, xv, yv, st, w_early); break;
            default: e = launch_nv<TYPE, 8>(tm, out_n, in_n, xv, yv, st, w_early); break;
        }
        if (e != cudaSuccess) return e;
        v0 += nv;
    }
    return cudaSuccess;
}

}  // namespace mvtc
