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
//     per vector so the largest |x| sits just below 2^15;
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

#include "pcu_common.cuh"

namespace mvtc {

constexpr int RT = 16;          // rows per tile (one MMA M)
constexpr int STAGES = 4;

enum : int { F_F16 = 1, F_Q4_0 = 2, F_Q8_0 = 8, F_Q4_K = 12, F_Q6_K = 14 };

// Per format: BE elements / BB bytes per block; SEGB blocks per stage;
// PITCH shared-memory bytes per row of a stage (the TMA box width: the
// stage's blocks plus a few bytes of the next ones, for bank spread);
// PERM: x stored as elements (0, 2, 1, 3) of every group of 4 (the order
// the nibble / byte unpacking produces); XSUM: per-32 sums of x kept;
// LOPAD: extra halves between a vector's hi and lo planes.
template <int TYPE> struct Fmt;
template <> struct Fmt<F_F16> {
    static constexpr int BE = 64, BB = 128, SEGB = 8, PITCH = 1056, PERM = 0, XSUM = 0, LOPAD = 16;
};
template <> struct Fmt<F_Q4_K> {
    static constexpr int BE = 256, BB = 144, SEGB = 8, PITCH = 1168, PERM = 1, XSUM = 1, LOPAD = 8;
};

// Consumer warps: 16 (four per SM sub-partition) while the registers of a
// thread allow it, 8 for the widest accumulator sets.
template <int NV> struct Warps {
    static constexpr int CW = NV <= 4 ? 16 : 8;
    static constexpr int THREADS = 32 * (CW + 1);
};

// Shared-memory layout; the x planes depend on in_n.
struct Smem {
    int stage, plane, lo, vstride, off_x, off_xsum, off_xinv, off_red, off_bar, bytes;
};
template <int TYPE>
__host__ __device__ inline Smem smem_layout(int in_n, int nv, int cw) {
    using F = Fmt<TYPE>;
    Smem s;
    s.stage = RT * F::PITCH;
    s.plane = ((in_n + in_n / 4) + 63) & ~63;          // halves, 8 bytes of pad per 16 elements
    s.lo = s.plane + F::LOPAD;
    s.vstride = (2 * s.plane + F::LOPAD + 63) & ~63;
    s.off_x = STAGES * s.stage;
    s.off_xsum = s.off_x + nv * s.vstride * 2;
    s.off_xinv = s.off_xsum + (F::XSUM ? nv * (in_n / 32) * 4 : 0);
    s.off_red = (s.off_xinv + 8 * 4 + 15) & ~15;       // also the x max scratch of the prologue
    s.off_bar = s.off_red + 2 * cw * RT * nv * 4;
    if (s.off_bar < s.off_red + 64 * 4) s.off_bar = s.off_red + 64 * 4;
    s.bytes = s.off_bar + 2 * STAGES * 8;
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

PCU_DEV uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
PCU_DEV uint2 lds64(const void* p) { return *reinterpret_cast<const uint2*>(p); }

// Byte `which` (0..3) of w as a float, exactly (0x4B000000 | b is 2^23 + b).
PCU_DEV float bytef(uint32_t w, int which) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440 | which)) - 8388608.0f;
}

PCU_DEV float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
PCU_DEV float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

PCU_DEV void wait_or_flag(uint64_t* bar, uint32_t parity, int code) {
    if (!mbar_wait(bar, parity)) record_error(&g_mv_err, code);
}

PCU_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// All threads: x [nv][in_n] into resident hi / lo planes, per-32 sums
// and each vector's 2^-s.
template <int TYPE, int NV, int THREADS>
PCU_DEV void convert_x(const float* __restrict__ x, int in_n, uint8_t* smem, const Smem& L) {
    using F = Fmt<TYPE>;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __half* xb = reinterpret_cast<__half*>(smem + L.off_x);
    float* xs = reinterpret_cast<float*>(smem + L.off_xsum);
    float* xi = reinterpret_cast<float*>(smem + L.off_xinv);
    float* scratch = reinterpret_cast<float*>(smem + L.off_red);
    #pragma unroll 1
    for (int v = 0; v < NV; ++v) {
        const float* xv = x + (size_t)v * in_n;
        float m = 0.f;
        for (int i = 4 * tid; i < in_n; i += 4 * THREADS) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(xv + i));
            m = fmaxf(m, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
        }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) scratch[warp] = m;
        __syncthreads();
        m = 0.f;
        for (int w = 0; w < THREADS / 32; ++w) m = fmaxf(m, scratch[w]);
        __syncthreads();
        int s = 14 - ((int)((__float_as_uint(m) >> 23) & 0xFF) - 127);
        s = max(-126, min(126, s));
        const float sc = __uint_as_float((uint32_t)(127 + s) << 23);
        __half* hp = xb + v * L.vstride;
        for (int i = 4 * tid; i < in_n; i += 4 * THREADS) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(xv + i));
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
            *reinterpret_cast<uint2*>(hp + xa(i)) = hv;
            *reinterpret_cast<uint2*>(hp + L.lo + xa(i)) = lv;
            if constexpr (F::XSUM != 0) {
                // in_n is a multiple of 256 here, so whole warps take part.
                float t = (q.x + q.y) + (q.z + q.w);
                t += __shfl_xor_sync(0xffffffffu, t, 1);
                t += __shfl_xor_sync(0xffffffffu, t, 2);
                t += __shfl_xor_sync(0xffffffffu, t, 4);
                if ((lane & 7) == 0) xs[v * (in_n / 32) + i / 32] = t;
            }
        }
        if (tid == 0) xi[v] = __uint_as_float((uint32_t)(127 - s) << 23);
    }
}

template <int TYPE, int NV>
__global__ void __launch_bounds__(Warps<NV>::THREADS, 1)
    matvec_tc_kernel(const __grid_constant__ CUtensorMap tm, int out_n, int in_n, const float* __restrict__ x,
                     float* __restrict__ y) {
    using F = Fmt<TYPE>;
    constexpr int CW = Warps<NV>::CW, THREADS = Warps<NV>::THREADS;
    extern __shared__ __align__(128) uint8_t smem[];
    const Smem L = smem_layout<TYPE>(in_n, NV, CW);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    uint64_t* b_full = bars;                 // [STAGES] TMA bytes landed
    uint64_t* b_empty = bars + STAGES;       // [STAGES] CW consumer warps done
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = in_n / F::BE;
    const int spt = (nb + F::SEGB - 1) / F::SEGB;                 // stages per tile
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

    // Stage s of this CTA: tile blockIdx.x + (s / spt) * gridDim.x, blocks
    // [(s % spt) * SEGB, +SEGB) of its rows.
    auto issue = [&](int s) {
        const int slot = s % STAGES;
        const int tile = (int)blockIdx.x + (s / spt) * (int)gridDim.x;
        mbar_arrive_expect_tx(&b_full[slot], (uint32_t)L.stage);
        tma_load_2d(smem + slot * L.stage, &tm, (s % spt) * (F::SEGB * F::BB / 8), tile * RT, &b_full[slot]);
    };
    if (warp == CW && lane == 0)
        for (int s = 0; s < min(STAGES, n_st); ++s) issue(s);
    convert_x<TYPE, NV, THREADS>(x, in_n, smem, L);
    __syncthreads();

    if (warp == CW) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            #pragma unroll 1
            for (int s = STAGES; s < n_st; ++s) {
                wait_or_flag(&b_empty[s % STAGES], ((s / STAGES) - 1) & 1, PCU_DEVERR_EMPTY_WAIT);
                issue(s);
            }
            // Every copy must have landed before the CTA may exit.
            for (int s = max(0, n_st - STAGES); s < n_st; ++s)
                wait_or_flag(&b_full[s % STAGES], (s / STAGES) & 1, PCU_DEVERR_DRAIN_WAIT);
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const bool act = (g >> 1) == t;                   // this lane's B fragment is non-zero
    const __half* xpl = reinterpret_cast<const __half*>(smem + L.off_x) + ((g & 1) ? L.lo : 0);
    const float* xsum = reinterpret_cast<const float*>(smem + L.off_xsum);
    const float* xinv = reinterpret_cast<const float*>(smem + L.off_xinv);
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    auto ldx = [&](int v, int h_off) -> uint2 {
        uint2 b = make_uint2(0u, 0u);
        if (act) b = lds64(xpl + v * L.vstride + h_off);
        return b;
    };
    float inv[NV];
    #pragma unroll
    for (int v = 0; v < NV; ++v) inv[v] = xinv[v];

    #pragma unroll 1
    for (int k = 0; k < my_tiles; ++k) {
        float acc[NV][2];
        #pragma unroll
        for (int v = 0; v < NV; ++v) acc[v][0] = acc[v][1] = 0.f;
        #pragma unroll 1
        for (int j = 0; j < spt; ++j) {
            const int s = k * spt + j, slot = s % STAGES;
            wait_or_flag(&b_full[slot], (s / STAGES) & 1, PCU_DEVERR_FULL_WAIT);
            const uint8_t* rows = smem + slot * L.stage;
            const int nblk = min(F::SEGB, nb - j * F::SEGB);
            #pragma unroll 1
            for (int bb = ((warp - j * F::SEGB) % CW + CW) % CW; bb < nblk; bb += CW) {
                const int e = (j * F::SEGB + bb) * F::BE;          // first element of the block
                if constexpr (TYPE == F_F16) {
                    // Block = 64 halves of a row; MMA i takes halves
                    // 16i + 4t .. +3 of rows g and g + 8 as lane (g, t)'s k slots.
                    const uint8_t* rg = rows + g * F::PITCH + bb * 128 + 8 * t;
                    const uint8_t* rg8 = rg + 8 * F::PITCH;
                    const int xb = xa(e + 4 * t);
                    float D[NV][4];
                    #pragma unroll
                    for (int v = 0; v < NV; ++v) D[v][0] = D[v][1] = D[v][2] = D[v][3] = 0.f;
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint2 a = lds64(rg + 32 * i), a8 = lds64(rg8 + 32 * i);
                        #pragma unroll
                        for (int v = 0; v < NV; ++v) mma16816(D[v], a.x, a8.x, a.y, a8.y, ldx(v, xb + 20 * i));
                    }
                    #pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        acc[v][0] += D[v][0] + D[v][1];
                        acc[v][1] += D[v][2] + D[v][3];
                    }
                } else if constexpr (TYPE == F_Q4_K) {
                    // Lane quad t takes chunk t (qs bytes 32t .. 32t+31) of the
                    // block: low nibbles = sub-block 2t, high nibbles = 2t + 1.
                    // Quants enter the MMA as 64 + q (exact f16); the 64 * sum(x)
                    // this adds comes off with the sub-block's x sum.
                    const uint8_t* bg = rows + g * F::PITCH + bb * 144;
                    const uint8_t* bg8 = bg + 8 * F::PITCH;
                    const uint4 qa = lds128(bg + 16 + 32 * t), qb = lds128(bg + 32 + 32 * t);
                    const uint4 qa8 = lds128(bg8 + 16 + 32 * t), qb8 = lds128(bg8 + 32 + 32 * t);
                    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    const uint32_t w8[8] = {qa8.x, qa8.y, qa8.z, qa8.w, qb8.x, qb8.y, qb8.z, qb8.w};
                    const int xb = xa(e + 64 * t);
                    float D[NV][2][4];
                    #pragma unroll
                    for (int v = 0; v < NV; ++v)
                        #pragma unroll
                        for (int q = 0; q < 4; ++q) D[v][0][q] = D[v][1][q] = 0.f;
                    constexpr uint32_t M = 0x00F000F0u, H64 = 0x54005400u;   // f16 64.0, ulp 1/16
                    #pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint32_t l0 = ((w[i] << 4) & M) | H64, l2 = ((w[i] >> 4) & M) | H64;
                        const uint32_t l1 = ((w8[i] << 4) & M) | H64, l3 = ((w8[i] >> 4) & M) | H64;
                        #pragma unroll
                        for (int v = 0; v < NV; ++v)
                            mma16816(D[v][0], l0, l1, l2, l3, ldx(v, xb + 4 * i + 4 * (i >> 2)));
                        const uint32_t h0 = (w[i] & M) | H64, h2 = ((w[i] >> 8) & M) | H64;
                        const uint32_t h1 = (w8[i] & M) | H64, h3 = ((w8[i] >> 8) & M) | H64;
                        #pragma unroll
                        for (int v = 0; v < NV; ++v)
                            mma16816(D[v][1], h0, h1, h2, h3, ldx(v, xb + 40 + 4 * i + 4 * (i >> 2)));
                    }
                    // Scales and mins of sub-blocks 2t, 2t + 1 (6-bit, packed in
                    // header bytes 4..15: src/pickle_fast.c:368-383).
                    const uint4 hg = lds128(bg), hg8 = lds128(bg8);
                    const int sh = 16 * (t & 1);
                    float ca[2], cb[2], da[2], db[2];
                    #pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const uint4 h = r ? hg8 : hg;
                        const uint32_t A1 = h.y >> sh, A2 = h.z >> sh, A3 = h.w >> sh;
                        const uint32_t sc2 = t < 2 ? (A1 & 0x3F3Fu) : ((A3 & 0x0F0Fu) | ((A1 >> 2) & 0x3030u));
                        const uint32_t m2 = t < 2 ? (A2 & 0x3F3Fu) : (((A3 >> 4) & 0x0F0Fu) | ((A2 >> 2) & 0x3030u));
                        const float d = h2f_lo(h.x), dmin = h2f_hi(h.x);
                        da[r] = d * bytef(sc2, 0);
                        db[r] = d * bytef(sc2, 1);
                        ca[r] = fmaf(64.f, da[r], dmin * bytef(m2, 0));
                        cb[r] = fmaf(64.f, db[r], dmin * bytef(m2, 1));
                    }
                    const int sub = e / 32 + 2 * t;
                    #pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float2 xs2 = *reinterpret_cast<const float2*>(xsum + v * (in_n / 32) + sub);
                        #pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            const float lo = D[v][0][2 * r] + D[v][0][2 * r + 1];
                            const float hi = D[v][1][2 * r] + D[v][1][2 * r + 1];
                            float a = acc[v][r];
                            a = fmaf(inv[v], fmaf(da[r], lo, db[r] * hi), a);
                            a = fmaf(-ca[r], xs2.x, a);
                            a = fmaf(-cb[r], xs2.y, a);
                            acc[v][r] = a;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&b_empty[slot]);
        }

        // Tile end: sum the lane quads, then the CW warps in a fixed order.
        float* rb = red + (k & 1) * CW * RT * NV;
        #pragma unroll
        for (int v = 0; v < NV; ++v)
            #pragma unroll
            for (int r = 0; r < 2; ++r) {
                float a = acc[v][r];
                a += __shfl_xor_sync(0xffffffffu, a, 1);
                a += __shfl_xor_sync(0xffffffffu, a, 2);
                if (t == 0) rb[(warp * RT + g + 8 * r) * NV + v] = a;
            }
        asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
        const int i = threadIdx.x;
        if (i < RT * NV) {
            const int r = i / NV, v = i % NV;
            float a = 0.f;
            for (int w = 0; w < CW; ++w) a += rb[(w * RT + r) * NV + v];
            const int row = ((int)blockIdx.x + k * (int)gridDim.x) * RT + r;
            if (row < out_n) y[(size_t)v * out_n + row] = TYPE == F_Q4_K ? a : a * xinv[v];
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

constexpr int kSmemLimit = 232448;

// True when the tensor-core path takes this call (otherwise the caller
// uses the CUDA-core kernel): 16-byte aligned rows, whole blocks, and x
// of one vector fitting in shared memory next to the ring.
template <int TYPE>
inline bool tc_supported(const void* W, size_t row_bytes, int in_n) {
    if (reinterpret_cast<uintptr_t>(W) % 16 || row_bytes % 16 || in_n % Fmt<TYPE>::BE) return false;
    if (Fmt<TYPE>::XSUM && in_n % 256) return false;
    return smem_layout<TYPE>(in_n, 1, Warps<1>::CW).bytes <= kSmemLimit;
}

template <int TYPE, int NV>
inline cudaError_t launch_nv(const CUtensorMap& tm, int out_n, int in_n, const float* x, float* y, cudaStream_t st) {
    const Smem L = smem_layout<TYPE>(in_n, NV, Warps<NV>::CW);
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
    matvec_tc_kernel<TYPE, NV><<<grid, Warps<NV>::THREADS, L.bytes, st>>>(tm, out_n, in_n, x, y);
    return cudaGetLastError();
}

template <int TYPE>
inline cudaError_t launch(const uint8_t* W, size_t row_bytes, int out_n, int in_n, int n_vec, const float* x,
                          float* y, cudaStream_t st) {
    alignas(64) CUtensorMap tm;
    if (make_w_map<TYPE>(&tm, W, row_bytes, out_n) != 0) return cudaErrorInvalidValue;
    // Vectors go in passes of as many as fit in shared memory.
    for (int v0 = 0; v0 < n_vec;) {
        int nv = n_vec - v0 < 8 ? n_vec - v0 : 8;
        while (nv > 1 && smem_layout<TYPE>(in_n, nv, nv <= 4 ? 16 : 8).bytes > kSmemLimit) --nv;
        const float* xv = x + (size_t)v0 * in_n;
        float* yv = y + (size_t)v0 * out_n;
        cudaError_t e = cudaSuccess;
        switch (nv) {
            case 1: e = launch_nv<TYPE, 1>(tm, out_n, in_n, xv, yv, st); break;
            case 2: e = launch_nv<TYPE, 2>(tm, out_n, in_n, xv, yv, st); break;
            case 3: e = launch_nv<TYPE, 3>(tm, out_n, in_n, xv, yv, st); break;
            case 4: e = launch_nv<TYPE, 4>(tm, out_n, in_n, xv, yv, st); break;
            case 5: e = launch_nv<TYPE, 5>(tm, out_n, in_n, xv, yv, st); break;
            case 6: e = launch_nv<TYPE, 6>(tm, out_n, in_n, xv, yv, st); break;
            case 7: e = launch_nv<TYPE, 7>(tm, out_n, in_n, xv, yv, st); break;
            default: e = launch_nv<TYPE, 8>(tm, out_n, in_n, xv, yv, st); break;
        }
        if (e != cudaSuccess) return e;
        v0 += nv;
    }
    return cudaSuccess;
}

}  // namespace mvtc
