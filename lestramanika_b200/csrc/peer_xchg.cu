// peer_xchg.cu - the exchange step of the sharded decodes over NVLink
// without NCCL: every rank writes its rows straight into every rank's
// receive buffer (plain peer stores through CUDA IPC mappings, no
// multicast) and the ranks meet on per-sender epoch flags.
//
// The two sharded decodes exchange little data per step (the 70B-shaped
// KV-head shard: 64 KiB per rank; the sequence-chunk shard: 16.6 KiB) and
// an NCCL all-gather plus the relayout of its output cost ~28 us of a
// 128 us step at 8 GPUs. Here one launch does it: CTA p serves rank p.
//   1. it takes this call's epoch e from its own counter slot (every CTA
//      runs once per call, so all slots agree, also across CUDA-graph
//      replays), publishes ready_p[rank] = e and waits until
//      ready_rank[p] == e: rank p has started its epoch-e call, so
//      everything that read rank p's buffer before (stream order) is done;
//   2. it copies this rank's rows into rank p's buffer at their final place
//      (so [B][H/N][D] head slices land directly as [B][H][D]);
//   3. it publishes done_p[rank] = e (system-scope release after a
//      system-scope fence) and waits until done_rank[p] == e: rank p's rows
//      have arrived here.
// Each rank's region is one cudaMalloc: the receive buffer, then the flag
// arrays (xchg_internal.cuh). Every wait is bounded (1 s by default,
// pickle_cuda_xchg_set_wait); giving up records an error that
// pickle_cuda_xchg_sync reports, and the exchange is then broken: the ranks'
// call counters no longer agree, so it must be recreated.
// The fused decode exchanges (pickle_cuda_decode_gather_dev,
// pickle_cuda_decode_seqshard_dev, in pickle_cuda.cu) use the same regions
// with per-row call counters and epoch-tagged data words.
#include "pickle_cuda.h"

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>

#include "pcu_common.cuh"
#include "xchg_internal.cuh"

namespace {

constexpr int kMaxRanks = kXchgMaxRanks;
constexpr int kPutThreads = 512;

struct PutArgs {
    unsigned char* peer_base[kMaxRanks];    // every rank's region, mapped here (own region for p == rank)
    size_t ready_off, done_off, epoch_off;   // byte offsets of the flag arrays in a region
    const unsigned char* src;
    size_t rows, row_bytes, src_stride, dst_offset, dst_stride;
    int rank, world;
    unsigned long long wait_ns;
    int* err;
};

PCU_DEV bool wait_flag(const unsigned* f, unsigned e, unsigned long long wait_ns) {
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_sys(f) != e)
        if (global_timer_ns() - t0 > wait_ns) return false;
    return true;
}

// CTA p: handshake with rank p, this rank's rows -> rank p's buffer, handshake again.
__global__ void __launch_bounds__(kPutThreads) xchg_put_kernel(const PutArgs a) {
    __shared__ int s_ok;
    const int p = blockIdx.x;
    unsigned char* mine = a.peer_base[a.rank];
    unsigned char* theirs = a.peer_base[p];
    unsigned e = 0;
    if (threadIdx.x == 0) {
        unsigned* slot = reinterpret_cast<unsigned*>(mine + a.epoch_off) + p;
        e = *slot + 1u;
        *slot = e;
        st_release_sys(reinterpret_cast<unsigned*>(theirs + a.ready_off) + a.rank, e);
        s_ok = wait_flag(reinterpret_cast<const unsigned*>(mine + a.ready_off) + p, e, a.wait_ns);
        if (!s_ok) record_error(a.err, PCU_DEVERR_FULL_WAIT);
    }
    __syncthreads();
    if (!s_ok) return;
    const size_t chunks = a.row_bytes / 16;
    for (size_t i = threadIdx.x; i < a.rows * chunks; i += blockDim.x) {
        const size_t r = i / chunks, c = i % chunks;
        const uint4 v = *reinterpret_cast<const uint4*>(a.src + r * a.src_stride + c * 16);
        *reinterpret_cast<uint4*>(theirs + a.dst_offset + r * a.dst_stride + c * 16) = v;
    }
    // Every thread's stores are ordered before the flag by the barrier and
    // the system-scope fence of the thread that publishes it.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<unsigned*>(theirs + a.done_off) + a.rank, e);
        if (!wait_flag(reinterpret_cast<const unsigned*>(mine + a.done_off) + p, e, a.wait_ns))
            record_error(a.err, PCU_DEVERR_FULL_WAIT);
    }
}

}  // namespace

extern "C" {

PICKLE_CUDA_API int pickle_cuda_xchg_create(int rank, int world, size_t buf_bytes, int device,
                                            pickle_cuda_xchg_t** out) {
    if (!out || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || buf_bytes == 0 ||
        buf_bytes % 16)
        return PICKLE_ERR_ARG;
    *out = nullptr;
    pickle_cuda_xchg* x = new (std::nothrow) pickle_cuda_xchg;
    if (!x) return PICKLE_ERR_MEMORY;
    x->rank = rank;
    x->world = world;
    x->device = device;
    x->buf_bytes = buf_bytes;
    x->ready_off = buf_bytes;
    x->done_off = x->ready_off + kMaxRanks * sizeof(unsigned);
    x->epoch_off = x->done_off + kMaxRanks * sizeof(unsigned);
    x->row_epoch_off = (buf_bytes + 256 + 255) / 256 * 256;
    x->region_bytes = x->row_epoch_off + (size_t)kXchgMaxRows * sizeof(unsigned);
    if (cudaSetDevice(device) != cudaSuccess || cudaMalloc(&x->region, x->region_bytes) != cudaSuccess ||
        cudaMemset(x->region, 0, x->region_bytes) != cudaSuccess ||
        cudaMalloc(&x->err_dev, sizeof(int)) != cudaSuccess || cudaMemset(x->err_dev, 0, sizeof(int)) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        pickle_cuda_xchg_free(x);
        return PICKLE_ERR_DEVICE;
    }
    x->peer[rank] = x->region;
    x->opened[rank] = true;
    *out = x;
    return PICKLE_OK;
}

PICKLE_CUDA_API int pickle_cuda_xchg_handle(pickle_cuda_xchg_t* x, void* handle_out) {
    if (!x || !handle_out) return PICKLE_ERR_ARG;
    cudaIpcMemHandle_t hnd;
    cudaError_t e = cudaIpcGetMemHandle(&hnd, x->region);
    if (e != cudaSuccess) {
        snprintf(x->last_error, sizeof(x->last_error), "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
        return PICKLE_ERR_DEVICE;
    }
    static_assert(sizeof(hnd) == PICKLE_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &hnd, sizeof(hnd));
    return PICKLE_OK;
}

PICKLE_CUDA_API int pickle_cuda_xchg_open(pickle_cuda_xchg_t* x, int peer, const void* handle) {
    if (!x || !handle || peer < 0 || peer >= x->world) return PICKLE_ERR_ARG;
    if (peer == x->rank || x->opened[peer]) return PICKLE_OK;
    cudaIpcMemHandle_t hnd;
    memcpy(&hnd, handle, sizeof(hnd));
    void* ptr = nullptr;
    cudaError_t e = cudaSetDevice(x->device);
    if (e == cudaSuccess) e = cudaIpcOpenMemHandle(&ptr, hnd, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        snprintf(x->last_error, sizeof(x->last_error), "cudaIpcOpenMemHandle(peer %d): %s", peer,
                 cudaGetErrorString(e));
        return PICKLE_ERR_DEVICE;
    }
    x->peer[peer] = static_cast<unsigned char*>(ptr);
    x->opened[peer] = true;
    x->ipc_mapped[peer] = true;
    return PICKLE_OK;
}

PICKLE_CUDA_API int pickle_cuda_xchg_attach(pickle_cuda_xchg_t* x, int peer, pickle_cuda_xchg_t* other) {
    if (!x || !other || peer < 0 || peer >= x->world || peer == x->rank || other->rank != peer ||
        other->world != x->world || other->buf_bytes != x->buf_bytes)
        return PICKLE_ERR_ARG;
    if (x->opened[peer]) return PICKLE_OK;
    if (other->device != x->device) {
        // Another GPU of this process: its memory must be reachable from ours.
        int can = 0;
        cudaError_t e = cudaDeviceCanAccessPeer(&can, x->device, other->device);
        if (e != cudaSuccess || !can) {
            snprintf(x->last_error, sizeof(x->last_error), "device %d cannot reach device %d", x->device,
                     other->device);
            return PICKLE_ERR_DEVICE;
        }
        e = cudaSetDevice(x->device);
        if (e == cudaSuccess) e = cudaDeviceEnablePeerAccess(other->device, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) {
            cudaGetLastError();
            e = cudaSuccess;
        }
        if (e != cudaSuccess) {
            snprintf(x->last_error, sizeof(x->last_error), "cudaDeviceEnablePeerAccess: %s", cudaGetErrorString(e));
            return PICKLE_ERR_DEVICE;
        }
    }
    x->peer[peer] = other->region;
    x->opened[peer] = true;
    return PICKLE_OK;
}

PICKLE_CUDA_API int pickle_cuda_xchg_set_wait(pickle_cuda_xchg_t* x, unsigned long long wait_ns) {
    if (!x || wait_ns == 0) return PICKLE_ERR_ARG;
    x->wait_ns = wait_ns;
    return PICKLE_OK;
}

PICKLE_CUDA_API int pickle_cuda_xchg_buffer(pickle_cuda_xchg_t* x, void** dev_ptr) {
    if (!x || !dev_ptr) return PICKLE_ERR_ARG;
    *dev_ptr = x->region;
    return PICKLE_OK;
}

PICKLE_CUDA_API int pickle_cuda_xchg_put_dev(pickle_cuda_xchg_t* x, const void* src, size_t rows, size_t row_bytes,
                                             size_t src_stride, size_t dst_offset, size_t dst_stride,
                                             void* stream) {
    if (!x || !src || rows == 0 || row_bytes == 0 || row_bytes % 16 || src_stride % 16 || dst_offset % 16 ||
        dst_stride % 16 || (uintptr_t)src % 16)
        return PICKLE_ERR_ARG;
    if (rows > 1 && (src_stride < row_bytes || dst_stride < row_bytes)) return PICKLE_ERR_ARG;
    if (dst_offset + (rows - 1) * dst_stride + row_bytes > x->buf_bytes) return PICKLE_ERR_RANGE;
    if (x->broken) {
        snprintf(x->last_error, sizeof(x->last_error), "exchange broken by an earlier wait that gave up: recreate it");
        return PICKLE_ERR_DEVICE;
    }
    for (int p = 0; p < x->world; ++p)
        if (!x->opened[p]) {
            snprintf(x->last_error, sizeof(x->last_error), "peer %d's region is not open", p);
            return PICKLE_ERR_ARG;
        }
    PutArgs a;
    memset(&a, 0, sizeof(a));
    for (int p = 0; p < x->world; ++p) a.peer_base[p] = x->peer[p];
    a.ready_off = x->ready_off;
    a.done_off = x->done_off;
    a.epoch_off = x->epoch_off;
    a.src = static_cast<const unsigned char*>(src);
    a.rows = rows;
    a.row_bytes = row_bytes;
    a.src_stride = rows > 1 ? src_stride : row_bytes;
    a.dst_offset = dst_offset;
    a.dst_stride = rows > 1 ? dst_stride : row_bytes;
    a.rank = x->rank;
    a.world = x->world;
    a.wait_ns = x->wait_ns;
    a.err = x->err_dev;
    xchg_put_kernel<<<x->world, kPutThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(x->last_error, sizeof(x->last_error), "xchg launch: %s", cudaGetErrorString(e));
        return PICKLE_ERR_DEVICE;
    }
    return PICKLE_OK;
}

PICKLE_CUDA_API int pickle_cuda_xchg_sync(pickle_cuda_xchg_t* x, void* stream) {
    if (!x) return PICKLE_ERR_ARG;
    int err = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&err, x->err_dev, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return PICKLE_ERR_DEVICE;
    if (err) {
        // The ranks' call counters no longer agree (this rank's moved on, a
        // peer's did not): every later call would wait in vain too.
        snprintf(x->last_error, sizeof(x->last_error),
                 "a peer never arrived (bounded wait gave up); the exchange is broken: recreate it");
        x->broken = true;
        cudaMemsetAsync(x->err_dev, 0, sizeof(int), st);
        cudaStreamSynchronize(st);
        return PICKLE_ERR_DEVICE;
    }
    return PICKLE_OK;
}

PICKLE_CUDA_API const char* pickle_cuda_xchg_last_error(pickle_cuda_xchg_t* x) {
    return x ? x->last_error : "null exchange";
}

PICKLE_CUDA_API void pickle_cuda_xchg_free(pickle_cuda_xchg_t* x) {
    if (!x) return;
    cudaSetDevice(x->device);
    cudaDeviceSynchronize();
    for (int p = 0; p < x->world; ++p)
        if (p != x->rank && x->ipc_mapped[p] && x->peer[p]) cudaIpcCloseMemHandle(x->peer[p]);
    cudaFree(x->region);
    cudaFree(x->err_dev);
    delete x;
}

}  // extern "C"
