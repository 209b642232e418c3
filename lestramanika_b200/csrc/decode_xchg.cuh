// decode_xchg.cuh - the split merge of the sharded decodes fused with their
// exchange over NVLink: one launch merges a rank's split partials, stores
// the result straight into every rank's receive buffer (plain peer stores
// through CUDA IPC mappings, no multicast), and assembles the final rows
// from what the other ranks stored, so the exchange costs no launch, no
// fence and no flag of its own.
//
// The reference decodes on one host (lee-muriithi-kingori/lestramanika
// src/pickle_fast.c:1946-2094, OpenMP over heads at :1960); the two shards
// split that block's work across GPUs:
//   gather (KV-head shard): CTA r merges output row r = (query z, local
//     head hl) of this rank's heads, normalised, and sends it to every rank;
//     it then writes row r of every rank p to out[z][p * n_heads + hl].
//   seqshard (sequence-chunk shard): CTA r merges the unnormalised triple
//     (M, L, acc[D]) of row r over this rank's cache chunk and sends it to
//     every rank; it then merges the triples of row r of all ranks by
//     log-sum-exp into out[r]:
//       M* = max_p M_p, o = sum_p e^(M_p - M*) acc_p / sum_p e^(M_p - M*) L_p.
//
// Wire format ("LL": each 8-byte word is 4 bytes of data and the 4-byte
// call epoch, written by one 16-byte store of two such words): a receiver
// polls the words themselves until every epoch field equals this call's e,
// so data and its arrival flag can never be seen apart and no memory fence
// is needed. Slot [half][sender][row] of the receive buffer, half = e & 1:
// a rank reaching call e + 2, which overwrites the half call e reads, has
// received every rank's rows of call e + 1, sent after their call e had
// finished reading. Epochs come from per-row counters in the own region,
// so CUDA-graph replays stay correct. Every wait is bounded (the exchange's
// wait limit); giving up records an error in the exchange's error word
// (pickle_cuda_xchg_sync) and the row is left unwritten.
#pragma once
#include "decode_splitkv.cuh"
#include "xchg_internal.cuh"

struct XchgMergeArgs {
    MergeArgs m;                     // this rank's split partials
    XchgPeers px;
    int mode;                        // 0: gather, 1: seqshard
    int n_rows;                      // rows of this rank (the grid)
    int rows_per_z;                  // gather: this rank's query heads per query
    unsigned long long row_bytes;    // one row's slot: D * 8 (gather), (D + 2) * 8 (seqshard)
    float* out;                      // gather: [n_z][world * rows_per_z][D]; seqshard: [n_rows][D]
    int* err;                        // the exchange's error word
};

// Two (data, epoch) words in one 16-byte store / load.
PCU_DEV void st_ll(unsigned char* p, float a, float b, unsigned e) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(__float_as_uint(a)), "r"(e),
                 "r"(__float_as_uint(b)), "r"(e)
                 : "memory");
}

// Poll two words at p until both carry epoch e; false after wait_ns.
PCU_DEV bool ld_ll(const unsigned char* p, unsigned e, unsigned long long wait_ns, float& a, float& b) {
    unsigned x, fx, y, fy;
    uint64_t t0 = 0;
    for (;;) {
        asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(x), "=r"(fx), "=r"(y), "=r"(fy)
                     : "l"(p)
                     : "memory");
        if (fx == e && fy == e) break;
        const uint64_t t = global_timer_ns();
        if (t0 == 0) t0 = t;
        else if (t - t0 > wait_ns) return false;
    }
    a = __uint_as_float(x);
    b = __uint_as_float(y);
    return true;
}

template <int D>
__global__ void __launch_bounds__(kMergeThreads) decode_merge_xchg_kernel(const XchgMergeArgs a) {
    constexpr int NCH = D / 4;
    __shared__ MergeSmem<D> sm;
    __shared__ unsigned s_e;
    __shared__ float s_m[kXchgMaxRanks], s_l[kXchgMaxRanks];
    __shared__ int s_ok;
    const int tid = threadIdx.x, row = blockIdx.x;
    const XchgPeers& px = a.px;
    unsigned char* own = px.base[px.rank];
    griddep_launch_dependents();                        // the next decode step's CTAs may become resident
    if (tid == 0) {
        unsigned* ep = reinterpret_cast<unsigned*>(own + px.row_epoch_off) + row;
        const unsigned e = *ep + 1u;
        *ep = e;
        s_e = e;
        s_ok = 1;
    }
    griddep_wait();                                     // the split kernel's partials are visible
    const float4 T = merge_splits<D>(a.m, row, sm);     // ends with a CTA barrier: s_e visible
    const unsigned e = s_e;
    const size_t half = (size_t)(e & 1u) * px.world * a.n_rows * a.row_bytes;
    // Send: this rank's row r into slot [half][rank][r] of every rank.
    const size_t my_slot = half + ((size_t)px.rank * a.n_rows + row) * a.row_bytes;
    if (tid < NCH) {
        float4 v = T;
        if (a.mode == 0) {
            const float inv = 1.0f / (sm.L == 0.0f ? 1.0f : sm.L);
            v = make_float4(T.x * inv, T.y * inv, T.z * inv, T.w * inv);
        }
        for (int p = 0; p < px.world; ++p) {
            unsigned char* dst = px.base[p] + my_slot + (size_t)tid * 32;
            st_ll(dst, v.x, v.y, e);
            st_ll(dst + 16, v.z, v.w, e);
        }
    } else if (tid == NCH && a.mode == 1) {
        for (int p = 0; p < px.world; ++p) st_ll(px.base[p] + my_slot + (size_t)D * 8, sm.M, sm.L, e);
    }
    // Receive row r of every rank.
    bool ok = true;
    if (a.mode == 0) {
        if (tid < NCH) {
            const int z = row / a.rows_per_z, hl = row % a.rows_per_z;
            for (int p = 0; p < px.world && ok; ++p) {
                const unsigned char* src = own + half + ((size_t)p * a.n_rows + row) * a.row_bytes + (size_t)tid * 32;
                float4 v;
                ok = ld_ll(src, e, px.wait_ns, v.x, v.y) && ld_ll(src + 16, e, px.wait_ns, v.z, v.w);
                if (ok) {
                    const size_t orow = ((size_t)z * px.world + p) * a.rows_per_z + hl;
                    reinterpret_cast<float4*>(a.out + orow * D)[tid] = v;
                }
            }
        }
        if (!ok) record_error(a.err, PCU_DEVERR_PEER_WAIT);
        return;
    }
    if (tid < px.world) {
        const unsigned char* src = own + half + ((size_t)tid * a.n_rows + row) * a.row_bytes + (size_t)D * 8;
        float mv = -INFINITY, lv = 0.f;
        if (!ld_ll(src, e, px.wait_ns, mv, lv)) s_ok = 0;
        s_m[tid] = mv;
        s_l[tid] = lv;
    }
    __syncthreads();
    if (!s_ok) {
        if (tid == 0) record_error(a.err, PCU_DEVERR_PEER_WAIT);
        return;
    }
    if (tid >= NCH) return;
    float M = -INFINITY;
    for (int p = 0; p < px.world; ++p) M = fmaxf(M, s_m[p]);
    float L = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < px.world && ok; ++p) {
        const unsigned char* src = own + half + ((size_t)p * a.n_rows + row) * a.row_bytes + (size_t)tid * 32;
        float4 x;
        ok = ld_ll(src, e, px.wait_ns, x.x, x.y) && ld_ll(src + 16, e, px.wait_ns, x.z, x.w);
        if (!ok || s_m[p] == -INFINITY) continue;
        const float w = expf(s_m[p] - M);
        L = fmaf(s_l[p], w, L);
        A.x = fmaf(w, x.x, A.x); A.y = fmaf(w, x.y, A.y);
        A.z = fmaf(w, x.z, A.z); A.w = fmaf(w, x.w, A.w);
    }
    if (!ok) {
        record_error(a.err, PCU_DEVERR_PEER_WAIT);
        return;
    }
    const float inv = 1.0f / (L == 0.0f ? 1.0f : L);
    reinterpret_cast<float4*>(a.out + (size_t)row * D)[tid] = make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv);
}

// Bytes of the receive buffer a fused exchange of n_rows rows per rank needs.
inline size_t decode_xchg_bytes(int mode, int world, int n_rows, int D) {
    const size_t row = (size_t)(mode == 0 ? D : D + 2) * 8;
    return 2 * (size_t)world * n_rows * row;
}

// Host: the fused merge launch, as a programmatic dependent of the split
// kernel just queued on `st`.
inline cudaError_t launch_decode_merge_xchg(int D, const XchgMergeArgs& x, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)x.n_rows);
    cfg.blockDim = dim3(kMergeThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (D) {
        case 48: return cudaLaunchKernelEx(&cfg, decode_merge_xchg_kernel<48>, x);
        case 64: return cudaLaunchKernelEx(&cfg, decode_merge_xchg_kernel<64>, x);
        case 96: return cudaLaunchKernelEx(&cfg, decode_merge_xchg_kernel<96>, x);
        case 128: return cudaLaunchKernelEx(&cfg, decode_merge_xchg_kernel<128>, x);
        case 256: return cudaLaunchKernelEx(&cfg, decode_merge_xchg_kernel<256>, x);
        default: return cudaErrorInvalidValue;
    }
}
