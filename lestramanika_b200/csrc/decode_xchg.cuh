// decode_xchg.cuh - the split merge of the sharded decodes fused with their
// exchange over NVLink: one launch merges a rank's split partials and
// stores the result straight into every rank's receive buffer (plain peer
// stores through CUDA IPC mappings, no multicast), so the exchange costs
// no launch and no local copy of its own.
//
// The reference decodes on one host (lee-muriithi-kingori/lestramanika
// src/pickle_fast.c:1946-2094, OpenMP over heads at :1960); the two shards
// split that block's work across GPUs:
//   gather (KV-head shard): CTA r merges output row r = (query z, local
//     head hl) of this rank's heads, normalised, and stores it at
//     dst_offset + z * dst_row_stride + hl * D * 4 in every rank's buffer,
//     i.e. straight into its place in [n_seqs][H][D];
//   seqshard (sequence-chunk shard): CTA r merges the unnormalised triple
//     (M, L, acc[D]) of row r over this rank's cache chunk, stores it into
//     slot [rank] of every rank's buffer, and once all ranks' triples of
//     row r have arrived merges them by log-sum-exp into out[r]:
//       M* = max_p M_p, o = sum_p e^(M_p - M*) acc_p / sum_p e^(M_p - M*) L_p.
//
// Per-row handshake (flags [sender][row] in each region, one counter per
// row in the own region, so CUDA-graph replays stay correct):
//   e = ++row_epoch[r];
//   gather: row_ready[rank][r] = e in every rank's region, before
//     griddepcontrol.wait: this rank has started the call, so what read its
//     buffer before (stream order) is done. The stores into rank p's
//     buffer wait until rank p's ready flag for row r has reached e.
//   seqshard: no ready flags. Calls alternate between two halves of the
//     buffer (parity of e). A rank reaching call e + 2, which writes the
//     half this call reads, has first seen this rank's done flag of call
//     e + 1, raised after this call finished reading.
//   Then, after a system-scope fence, row_done[rank][r] = e in every
//   rank's region, and the CTA waits until every rank's done flag for row
//   r has reached e: all rows r have arrived here.
// Every wait is bounded (the exchange's wait limit); giving up records an
// error in the exchange's error word (pickle_cuda_xchg_sync) and the CTA
// skips what depends on it.
#pragma once
#include "decode_splitkv.cuh"
#include "xchg_internal.cuh"

struct XchgMergeArgs {
    MergeArgs m;                     // this rank's split partials
    XchgPeers px;
    int mode;                        // 0: gather, 1: seqshard
    int n_rows;                      // rows of this rank (the grid)
    int rows_per_z;                  // gather: this rank's query heads per query
    unsigned long long dst_offset;   // gather: bytes
    unsigned long long dst_row_stride;
    unsigned long long part_bytes;   // seqshard: one rank's slot: rows * (D + 2) * 4, 16-byte multiple
    float* out;                      // seqshard: merged rows [n_rows][D] (local)
    int* err;                        // the exchange's error word
};

template <int D>
__global__ void __launch_bounds__(kMergeThreads) decode_merge_xchg_kernel(const XchgMergeArgs a) {
    constexpr int NCH = D / 4;
    __shared__ MergeSmem<D> sm;
    __shared__ unsigned s_e;
    __shared__ int s_ok;
    const int tid = threadIdx.x, row = blockIdx.x;
    const XchgPeers& px = a.px;
    unsigned char* own = px.base[px.rank];
    if (tid == 0) {
        unsigned* ep = reinterpret_cast<unsigned*>(own + px.row_epoch_off) + row;
        const unsigned e = *ep + 1u;
        *ep = e;
        s_e = e;
        s_ok = 1;
        if (a.mode == 0)
            for (int p = 0; p < px.world; ++p) st_release_sys(row_flag(px.base[p], px.row_ready_off, px.rank, row), e);
    }
    griddep_wait();                                     // the split kernel's partials are visible
    const float4 T = merge_splits<D>(a.m, row, sm);     // ends with a CTA barrier: s_e, s_ok visible
    const unsigned e = s_e;
    const int parity = (int)(e & 1u);
    if (a.mode == 0) {
        if (tid == 0) {
            for (int p = 0; p < px.world && s_ok; ++p)
                s_ok = wait_epoch(row_flag(own, px.row_ready_off, p, row), e, px.wait_ns);
        }
        __syncthreads();
        if (s_ok && tid < NCH) {
            const float inv = 1.0f / (sm.L == 0.0f ? 1.0f : sm.L);
            const float4 v = make_float4(T.x * inv, T.y * inv, T.z * inv, T.w * inv);
            const int z = row / a.rows_per_z, hl = row % a.rows_per_z;
            const size_t off = a.dst_offset + (size_t)z * a.dst_row_stride + ((size_t)hl * D + 4 * tid) * 4;
            for (int p = 0; p < px.world; ++p) *reinterpret_cast<float4*>(px.base[p] + off) = v;
        }
    } else {
        const size_t slot = ((size_t)parity * px.world + px.rank) * a.part_bytes;
        if (tid < NCH)
            for (int p = 0; p < px.world; ++p)
                reinterpret_cast<float4*>(px.base[p] + slot + (size_t)row * D * 4)[tid] = T;
        if (tid == 0)
            for (int p = 0; p < px.world; ++p) {
                float* ml = reinterpret_cast<float*>(px.base[p] + slot + (size_t)a.n_rows * D * 4);
                ml[row] = sm.M;
                ml[a.n_rows + row] = sm.L;
            }
    }
    // Every thread's stores are ordered before the done flags by the barrier
    // and the system-scope fence of the thread that publishes them.
    __syncthreads();
    if (tid == 0) {
        if (s_ok) {
            __threadfence_system();
            for (int p = 0; p < px.world; ++p) st_release_sys(row_flag(px.base[p], px.row_done_off, px.rank, row), e);
            for (int p = 0; p < px.world && s_ok; ++p)
                s_ok = wait_epoch(row_flag(own, px.row_done_off, p, row), e, px.wait_ns);
        }
        if (!s_ok) record_error(a.err, PCU_DEVERR_PEER_WAIT);
    }
    __syncthreads();
    if (a.mode != 1 || !s_ok || tid >= NCH) return;
    // Log-sum-exp merge of the world triples of row r, read past L1 (other
    // GPUs wrote them).
    const unsigned char* half = own + (size_t)parity * px.world * a.part_bytes;
    float mp[kXchgMaxRanks];
    float M = -INFINITY;
    for (int p = 0; p < px.world; ++p) {
        mp[p] = __ldcg(reinterpret_cast<const float*>(half + p * a.part_bytes + (size_t)a.n_rows * D * 4) + row);
        M = fmaxf(M, mp[p]);
    }
    float L = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < px.world; ++p) {
        if (mp[p] == -INFINITY) continue;
        const unsigned char* part = half + p * a.part_bytes;
        const float w = expf(mp[p] - M);
        L = fmaf(__ldcg(reinterpret_cast<const float*>(part + (size_t)a.n_rows * D * 4) + a.n_rows + row), w, L);
        const float4 x = __ldcg(reinterpret_cast<const float4*>(part + (size_t)row * D * 4) + tid);
        A.x = fmaf(w, x.x, A.x); A.y = fmaf(w, x.y, A.y);
        A.z = fmaf(w, x.z, A.z); A.w = fmaf(w, x.w, A.w);
    }
    const float inv = 1.0f / (L == 0.0f ? 1.0f : L);
    reinterpret_cast<float4*>(a.out + (size_t)row * D)[tid] = make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv);
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
