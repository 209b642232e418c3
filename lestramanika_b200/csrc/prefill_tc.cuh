// prefill_tc.cuh - causal prefill attention on the sm_100a tensor cores.
//
// Replaces the reference's token-by-token prefill
// (lee-muriithi-kingori/lestramanika src/pickle_fast.c:1881 over
// :1946-2094): for every query position t of the prompt, softmax over
// keys [0, t] of q_t . k / sqrtf(D), weighted sum of V, per query head with
// kv_head = h * HK / H. Operands are BF16 copies of the rotated q/k/v
// (written by rope_append_kernel), accumulation is F32 in tensor memory,
// the output is F32.
//
// One CTA owns a 128-row query tile of one (sequence, head):
//   warp 4      one lane loads Q once and K/V tiles (128 keys) into a
//               2-stage ring with 3-D TMA tensor copies (128-byte swizzle,
//               no multicast);
//   warp 5      allocates 512 TMEM columns and one lane issues tcgen05.mma:
//               S_j = Q K_j^T into one of two S buffers (M=N=128, K=D), then
//               O += P_{j-1} V_{j-1} (A = P from shared memory, B = V read
//               MN-major), committing to mbarriers;
//   warps 0-3   the softmax warpgroup: thread r owns query row r, reads its
//               S row from TMEM (tcgen05.ld), applies the causal mask, keeps
//               the running max in the log2 domain (rescaling O in TMEM only
//               when the max grows by more than 2^8), writes P as BF16 into
//               the swizzled K-major layout the MMA reads, and at the end
//               normalises its O row and stores it.
// S_{j+1} is computed by the tensor cores while the softmax works on S_j.
// Every mbarrier wait is bounded; a timeout sets the error word, drains the
// copies and MMAs in flight, frees TMEM and exits.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>

#include "pcu_common.cuh"

namespace tc {

constexpr int BM = 128;                    // query rows per CTA
constexpr int BN = 128;                    // keys per tile
constexpr int HD = 128;                    // head dim handled here
constexpr int HALF_BYTES = 128 * 128;      // one 64-column half of a 128-row tile (bf16)
constexpr int TILE_BYTES = 2 * HALF_BYTES; // 128 x 128 bf16
constexpr int STAGES = 2;
constexpr int SMEM_Q = 0;
constexpr int SMEM_KV = SMEM_Q + TILE_BYTES;                 // stage s: K at +2s*TILE, V at +(2s+1)*TILE
constexpr int SMEM_P = SMEM_KV + STAGES * 2 * TILE_BYTES;
constexpr int SMEM_BAR = SMEM_P + TILE_BYTES;
constexpr int N_BARS = 16;
constexpr int SMEM_BYTES = SMEM_BAR + N_BARS * 8 + 16 + 1024; // + TMEM address slot + alignment slack
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

// Barrier slots.
enum { B_Q = 0, B_KV_FULL = 1, B_KV_EMPTY = 3, B_S_FULL = 5, B_S_FREE = 7, B_P_FULL = 9, B_PV_DONE = 10,
       B_DRAIN = 11 };

// tcgen05 instruction descriptor, kind::f16: F32 accumulate, BF16 A and B,
// M = 128, N = 128, A K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1).
__host__ __device__ constexpr uint32_t idesc_bf16(int n, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version bits.
PCU_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

PCU_DEV void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

PCU_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

PCU_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

PCU_DEV void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

PCU_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

PCU_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PCU_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
PCU_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive 32-bit columns of this thread's TMEM lane. The wait is in
// the same asm statement, so no use of the outputs can be scheduled before
// the load has landed in the registers.
PCU_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
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

PCU_DEV void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
          "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
          "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
          "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
          "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
          "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
          "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
          "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
          "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
          "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
          "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

PCU_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

PCU_DEV uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

struct PrefillTcArgs {
    float* ao;            // [n_seqs][T][H][D] F32
    int T, H, HK, n_qt;
    float scale_log2;     // log2(e) / sqrtf(D)
    int* err;
};

__global__ void __launch_bounds__(THREADS, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const PrefillTcArgs a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned base (128-byte swizzle atoms).
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_u32 - raw_u32);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + SMEM_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + SMEM_BAR + N_BARS * 8);
    __shared__ int s_abort, s_issued;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, seq = blockIdx.y;
    const int qt = a.n_qt - 1 - (int)blockIdx.z;           // heaviest query tiles first
    const int q0 = qt * BM;
    const int kvh = h * a.HK / a.H;                         // src/pickle_fast.c:1963
    const int n_kv = min((q0 + BM + BN - 1) / BN, (a.T + BN - 1) / BN);

    if (tid == 0) {
        mbar_init(&bars[B_Q], 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars[B_KV_FULL + s], 1);
            mbar_init(&bars[B_KV_EMPTY + s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[B_S_FULL + b], 1);
            mbar_init(&bars[B_S_FREE + b], 4);
        }
        mbar_init(&bars[B_P_FULL], 4);
        mbar_init(&bars[B_PV_DONE], 1);
        mbar_init(&bars[B_DRAIN], 1);
        mbar_fence_init();
        s_abort = 0;
        s_issued = 0;
    }
    if (warp == 5) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_S0 = tmem, tmem_O = tmem + 256;

    if (warp == 4) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const int zq = seq * a.H + h, zk = seq * a.HK + kvh;
            mbar_arrive_expect_tx(&bars[B_Q], TILE_BYTES);
            tma_load_3d(base_u32 + SMEM_Q, &tm_q, 0, q0, zq, &bars[B_Q]);
            tma_load_3d(base_u32 + SMEM_Q + HALF_BYTES, &tm_q, 64, q0, zq, &bars[B_Q]);
            for (int j = 0; j < n_kv; ++j) {
                const int s = j % STAGES;
                if (j >= STAGES && !mbar_wait(&bars[B_KV_EMPTY + s], ((j / STAGES) - 1) & 1)) {
                    record_error(a.err, PCU_DEVERR_EMPTY_WAIT);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int*)&s_abort) break;
                const uint32_t kdst = base_u32 + SMEM_KV + (2 * s) * TILE_BYTES;
                const uint32_t vdst = kdst + TILE_BYTES;
                mbar_arrive_expect_tx(&bars[B_KV_FULL + s], 2 * TILE_BYTES);
                tma_load_3d(kdst, &tm_k, 0, j * BN, zk, &bars[B_KV_FULL + s]);
                tma_load_3d(kdst + HALF_BYTES, &tm_k, 64, j * BN, zk, &bars[B_KV_FULL + s]);
                tma_load_3d(vdst, &tm_v, 0, j * BN, zk, &bars[B_KV_FULL + s]);
                tma_load_3d(vdst + HALF_BYTES, &tm_v, 64, j * BN, zk, &bars[B_KV_FULL + s]);
                s_issued = j + 1;
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t id_qk = idesc_bf16(BN, 0);
            const uint32_t id_pv = idesc_bf16(HD, 1);
            bool ok = mbar_wait(&bars[B_Q], 0);
            tc_fence_after();
            for (int j = 0; ok && j <= n_kv; ++j) {
                if (j < n_kv) {
                    const int s = j % STAGES, b = j & 1;
                    ok = mbar_wait(&bars[B_KV_FULL + s], (j / STAGES) & 1);
                    if (ok && j >= 2) ok = mbar_wait(&bars[B_S_FREE + b], ((j / 2) - 1) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t kaddr = base_u32 + SMEM_KV + (2 * s) * TILE_BYTES;
                    #pragma unroll
                    for (int ks = 0; ks < HD / 16; ++ks) {
                        const uint32_t off = (ks / 4) * HALF_BYTES + (ks % 4) * 32;
                        mma_bf16(tmem_S0 + b * 128, smem_desc(base_u32 + SMEM_Q + off, 16, 1024),
                                 smem_desc(kaddr + off, 16, 1024), id_qk, ks > 0);
                    }
                    mma_commit(&bars[B_S_FULL + b]);
                }
                if (j >= 1) {
                    const int jp = j - 1, s = jp % STAGES;
                    ok = mbar_wait(&bars[B_P_FULL], jp & 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t vaddr = base_u32 + SMEM_KV + (2 * s + 1) * TILE_BYTES;
                    #pragma unroll
                    for (int ks = 0; ks < BN / 16; ++ks) {
                        const uint32_t poff = (ks / 4) * HALF_BYTES + (ks % 4) * 32;
                        mma_bf16(tmem_O, smem_desc(base_u32 + SMEM_P + poff, 16, 1024),
                                 smem_desc(vaddr + ks * 16 * 128, HALF_BYTES, 1024), id_pv, (jp > 0 || ks > 0));
                    }
                    mma_commit(&bars[B_PV_DONE]);
                    mma_commit(&bars[B_KV_EMPTY + s]);
                }
            }
            if (!ok) {
                record_error(a.err, PCU_DEVERR_MMA_WAIT);
                s_abort = 1;
            }
            // Let every MMA this thread issued finish before TMEM can be freed.
            mma_commit(&bars[B_DRAIN]);
            if (!mbar_wait(&bars[B_DRAIN], 0)) record_error(a.err, PCU_DEVERR_DRAIN_WAIT);
        }
    } else {
        // ---------------- softmax warpgroup: thread = query row ----------------
        const int row = tid;                                  // 0..127 (TMEM lane)
        const int q = q0 + row;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        unsigned char* pbase = base + SMEM_P;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int b = j & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_S_FULL + b], (j / 2) & 1));
            if (!ok) break;
            tc_fence_after();
            float s[BN];
            #pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
                float v[32];
                tmem_ld32(tmem_S0 + b * 128 + lane_off + c * 32, v);
                #pragma unroll
                for (int i = 0; i < 32; ++i) s[c * 32 + i] = v[i];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_S_FREE + b]);
            // causal mask (and keys past T on a ragged last tile)
            const int k0 = j * BN;
            if (k0 + BN - 1 > q0 || k0 + BN > a.T) {
                #pragma unroll
                for (int c = 0; c < BN; ++c)
                    if (k0 + c > q || k0 + c >= a.T) s[c] = -INFINITY;
            }
            float mx = -INFINITY;
            #pragma unroll
            for (int c = 0; c < BN; ++c) mx = fmaxf(mx, s[c]);
            const float m_tile = mx * a.scale_log2;
            float alpha = 1.0f;
            const bool grow = m_tile > m_run + RESCALE_THRESHOLD || m_run == -INFINITY;
            if (grow) {
                alpha = exp2f(m_run - m_tile);
                m_run = m_tile;
            }
            float sum = 0.f;
            #pragma unroll
            for (int c = 0; c < BN; ++c) {
                s[c] = exp2f(fmaf(s[c], a.scale_log2, -m_run));
                sum += s[c];
            }
            // P buffer and O are owned by PV_{j-1} until it completes.
            if (j >= 1) {
                ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_PV_DONE], (j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
                if (__any_sync(0xffffffffu, grow)) {
                    #pragma unroll
                    for (int c = 0; c < HD / 32; ++c) {
                        float o[32];
                        tmem_ld32(tmem_O + lane_off + c * 32, o);
                        #pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(tmem_O + lane_off + c * 32, o);
                    }
                    tmem_st_wait();
                }
            }
            l_run = l_run * alpha + sum;
            // P row -> 128-byte-swizzled K-major tile (two 64-key halves).
            #pragma unroll
            for (int ch = 0; ch < BN / 8; ++ch) {
                const int half = ch / 8, chunk = ch % 8;
                uint4 w;
                w.x = pack_bf16x2(s[ch * 8 + 0], s[ch * 8 + 1]);
                w.y = pack_bf16x2(s[ch * 8 + 2], s[ch * 8 + 3]);
                w.z = pack_bf16x2(s[ch * 8 + 4], s[ch * 8 + 5]);
                w.w = pack_bf16x2(s[ch * 8 + 6], s[ch * 8 + 7]);
                const int off = half * HALF_BYTES + (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
                *reinterpret_cast<uint4*>(pbase + off) = w;
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_P_FULL]);
        }
        if (ok && n_kv > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_PV_DONE], (n_kv - 1) & 1));
        if (!ok) {
            if (lane == 0) { record_error(a.err, PCU_DEVERR_FULL_WAIT); s_abort = 1; }
        } else {
            tc_fence_after();
            const float inv = 1.0f / (l_run == 0.0f ? 1.0f : l_run);
            float* orow = a.ao + (((size_t)seq * a.T + q) * a.H + h) * HD;
            #pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                float o[32];
                tmem_ld32(tmem_O + lane_off + c * 32, o);
                if (q < a.T) {
                    #pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(orow + c * 32 + i) =
                            make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4 && lane == 0 && s_abort) {
        // Copies issued but never consumed must land before shared memory goes away:
        // the last STAGES tiles issued cover every copy that can still be in flight.
        const int issued = s_issued;
        for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
            if (!mbar_wait(&bars[B_KV_FULL + j % STAGES], (j / STAGES) & 1)) record_error(a.err, PCU_DEVERR_DRAIN_WAIT);
        if (!mbar_wait(&bars[B_Q], 0)) record_error(a.err, PCU_DEVERR_DRAIN_WAIT);
    }
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace tc

inline bool prefill_tc_supported(int D, int G) { return D == tc::HD && G >= 1 && G <= 8; }

// 3-D tensor map over a head-major BF16 tensor [n_heads][T][D]: box 64 x 128 x 1.
inline int make_tmap(CUtensorMap* map, const void* ptr, int T, int n_heads, char* msg, size_t msg_len) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn) {
            snprintf(msg, msg_len, "cuTensorMapEncodeTiled not available");
            return -9;
        }
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[3] = {(cuuint64_t)tc::HD, (cuuint64_t)T, (cuuint64_t)n_heads};
    const cuuint64_t strides[2] = {(cuuint64_t)tc::HD * 2, (cuuint64_t)T * tc::HD * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)tc::BM, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(msg, msg_len, "cuTensorMapEncodeTiled failed (%d)", (int)r);
        return -9;
    }
    return 0;
}

// q: [n_seqs][H][T][D], k/v: [n_seqs][HK][T][D] BF16 (rotated); ao: [n_seqs][T][H][D] F32.
inline int prefill_tc_launch(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, float* ao,
                             int n_seqs, int T, int H, int HK, int D, float scale, int* err, cudaStream_t st,
                             char* msg, size_t msg_len) {
    if (D != tc::HD) {
        snprintf(msg, msg_len, "tensor-core prefill needs head_dim %d", tc::HD);
        return -6;
    }
    alignas(64) CUtensorMap tq, tk, tv;
    if (make_tmap(&tq, q, T, n_seqs * H, msg, msg_len) || make_tmap(&tk, k, T, n_seqs * HK, msg, msg_len) ||
        make_tmap(&tv, v, T, n_seqs * HK, msg, msg_len))
        return -9;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(tc::prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             tc::SMEM_BYTES);
        if (e != cudaSuccess) {
            snprintf(msg, msg_len, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return -9;
        }
        attr_set = true;
    }
    tc::PrefillTcArgs a;
    a.ao = ao;
    a.T = T;
    a.H = H;
    a.HK = HK;
    a.n_qt = (T + tc::BM - 1) / tc::BM;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.err = err;
    dim3 grid((unsigned)H, (unsigned)n_seqs, (unsigned)a.n_qt);
    tc::prefill_tc_kernel<<<grid, tc::THREADS, tc::SMEM_BYTES, st>>>(tq, tk, tv, a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(msg, msg_len, "prefill_tc launch: %s", cudaGetErrorString(e));
        return -9;
    }
    return 0;
}
