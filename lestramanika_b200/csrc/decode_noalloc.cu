// decode_noalloc.cu - the split-KV decode for callers that cannot allocate
// device memory.
//
// Some hosts of this attention block own all of the GPU's memory through
// their own arena: an engine that reserves HBM for its KV cache up front
// and hands out slices, or a pickle build whose every allocation must go
// through its pickle_alloc_t callbacks. Such a caller can pass us device
// buffers it already owns, but it cannot let a library call cudaMalloc
// behind its back. pickle_cuda_decode_noalloc therefore takes every input
// and output from the caller (q, k, v, the KV cache, the RoPE tables, ao)
// and keeps its only scratch - the split-KV partial results - in one
// fixed array below.
//
// The array is a file-scope __device__ object of kNoAllocScratchBytes
// (4 MiB); every GPU that loads this library holds it until the process
// exits. All calls share it, so calls whose kernels overlap on the GPU
// (other streams, other host threads) race on the array - serialise them
// on one stream. A call is two launches (split kernel, then the merge
// kernel as its programmatic dependent) when it plans several splits.
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress (host code may not use the symbol itself as a
// device pointer), and the first call with each head dim and GQA group
// size sets that kernel's shared-memory limit and queries its occupancy;
// make those first calls before any stream capture. Later calls reuse the
// cached values without taking a lock.
#include "pickle_cuda.h"

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "decode_splitkv.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;          // 4 MiB
constexpr int kNoAllocMaxGroups = 4096;                     // n_seqs * n_kv_heads
constexpr int kNoAllocMaxDevices = 64;

// Layout: [partials: m rows, l rows, acc rows].
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocKernels = 5 * 4;                      // head dims x GQA group sizes

// Set up once per device under the mutex; later calls read it without the
// lock (ready and occ[] are published with release stores after the fields
// they guard).
struct NoAllocDevice {
    std::atomic<bool> ready{false};
    unsigned char* scratch = nullptr;     // device address of g_noalloc_scratch
    int num_sms = 0;
    std::atomic<int> occ[kNoAllocKernels] = {};   // resident CTAs per SM of each kernel; 0: not prepared
};
NoAllocDevice g_dev[kNoAllocMaxDevices];
std::mutex g_dev_mutex;

struct NoAllocKernel {
    const void* fn;
    int threads;
    size_t smem;
    int tile_rows;
    int index;                            // slot in NoAllocDevice::occ
};

template <int D, int G>
NoAllocKernel noalloc_kernel() {
    using C = DecodeCfg<D, G>;
    const int di = D == 48 ? 0 : D == 64 ? 1 : D == 96 ? 2 : D == 128 ? 3 : 4;
    const int gi = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
    return {reinterpret_cast<const void*>(&decode_splitkv_kernel<D, G>), C::THREADS, C::SMEM, C::TP, di * 4 + gi};
}

template <int D>
bool noalloc_pick_g(int G, NoAllocKernel* k) {
    switch (G) {
        case 1: *k = noalloc_kernel<D, 1>(); return true;
        case 2: *k = noalloc_kernel<D, 2>(); return true;
        case 4: *k = noalloc_kernel<D, 4>(); return true;
        case 8: *k = noalloc_kernel<D, 8>(); return true;
        default: return false;
    }
}

bool noalloc_pick(int D, int G, NoAllocKernel* k) {
    switch (D) {
        case 48: return noalloc_pick_g<48>(G, k);
        case 64: return noalloc_pick_g<64>(G, k);
        case 96: return noalloc_pick_g<96>(G, k);
        case 128: return noalloc_pick_g<128>(G, k);
        case 256: return noalloc_pick_g<256>(G, k);
        default: return false;
    }
}

void report(const char* what, cudaError_t e) {
    fprintf(stderr, "pickle_cuda_decode_noalloc: %s: %s\n", what, cudaGetErrorString(e));
}

// Once per device, with that device current: the scratch address and the
// SM count; once per (device, kernel): the kernel's shared-memory limit and
// its occupancy. Later calls take the cached values without the lock.
int noalloc_setup(int device, const NoAllocKernel& k, NoAllocDevice** out, int* occ_out) {
    if (device < 0 || device >= kNoAllocMaxDevices) return PICKLE_ERR_ARG;
    NoAllocDevice& d = g_dev[device];
    int occ = d.ready.load(std::memory_order_acquire) ? d.occ[k.index].load(std::memory_order_acquire) : 0;
    if (occ < 1) {
        std::lock_guard<std::mutex> lock(g_dev_mutex);
        if (!d.ready.load(std::memory_order_relaxed)) {
            void* ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess) { report("cudaGetSymbolAddress", e); return PICKLE_ERR_DEVICE; }
            e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device);
            if (e != cudaSuccess) { report("cudaDeviceGetAttribute", e); return PICKLE_ERR_DEVICE; }
            d.scratch = static_cast<unsigned char*>(ptr);
            d.ready.store(true, std::memory_order_release);
        }
        occ = d.occ[k.index].load(std::memory_order_relaxed);
        if (occ < 1) {
            cudaError_t e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)k.smem);
            if (e != cudaSuccess) { report("cudaFuncSetAttribute", e); return PICKLE_ERR_DEVICE; }
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k.fn, k.threads, k.smem);
            if (e != cudaSuccess || occ < 1) { report("occupancy", e); return PICKLE_ERR_DEVICE; }
            d.occ[k.index].store(occ, std::memory_order_release);
        }
    }
    *out = &d;
    *occ_out = occ;
    return PICKLE_OK;
}

}  // namespace

extern "C" PICKLE_CUDA_API int pickle_cuda_decode_noalloc(
    int n_seqs, int n_heads, int n_kv_heads, int head_dim, int half, int max_seq, size_t pos,
    const float* rope_sin, const float* rope_cos, const float* q, const float* k, const float* v,
    float* k_cache, float* v_cache, float* ao, int* err_flag, void* stream) {
    if (n_seqs < 1 || n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads || head_dim % 4 ||
        half < 0 || 2 * half > head_dim || max_seq < 1 || !rope_sin || !rope_cos || !q || !k || !v ||
        !k_cache || !v_cache || !ao)
        return PICKLE_ERR_ARG;
    // Rows move as 16-byte vectors and bulk copies: every row pointer must be 16-byte aligned.
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)k_cache | (uintptr_t)v_cache |
         (uintptr_t)ao) % 16)
        return PICKLE_ERR_ARG;
    if (pos >= (size_t)max_seq) return PICKLE_ERR_RANGE;
    const int G = n_heads / n_kv_heads;
    NoAllocKernel kern;
    if (!noalloc_pick(head_dim, G, &kern)) return PICKLE_ERR_ARG;
    const long long groups = (long long)n_seqs * n_kv_heads;
    if (groups > kNoAllocMaxGroups) {
        fprintf(stderr, "pickle_cuda_decode_noalloc: n_seqs * n_kv_heads = %lld exceeds the %d "
                        "sequence/KV-head slots of the %zu-byte scratch array\n",
                groups, kNoAllocMaxGroups, kNoAllocScratchBytes);
        return PICKLE_ERR_RANGE;
    }
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) { report("cudaGetDevice", e); return PICKLE_ERR_DEVICE; }
    NoAllocDevice* dev = nullptr;
    int occ = 0;
    int rc = noalloc_setup(device, kern, &dev, &occ);
    if (rc != PICKLE_OK) return rc;

    // Split plan: fill the SMs, but never more partial rows than the array holds.
    const size_t row_bytes = (size_t)(head_dim + 2) * sizeof(float);
    const long long row_cap = (long long)((kNoAllocScratchBytes - 64) / row_bytes);
    const long long hist = (long long)pos;
    int n_splits = 1;
    if (hist > 0) {
        const long long slots = (long long)dev->num_sms * occ;
        long long max_s = hist / (2 * kern.tile_rows);
        if (max_s > kMaxSplits) max_s = kMaxSplits;
        const long long cap = row_cap / (groups * G);
        if (max_s > cap) max_s = cap;
        n_splits = plan_decode_splits(groups, hist, slots, max_s, G, head_dim);
    }
    const size_t part_rows = (size_t)groups * G * n_splits;

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* base = dev->scratch;
    const size_t part_rows4 = (part_rows + 3) & ~size_t(3);   // keeps ws_acc 16-byte aligned
    float* ws_m = reinterpret_cast<float*>(base);
    float* ws_l = ws_m + part_rows4;
    float* ws_acc = ws_l + part_rows4;

    DecodeArgs a;
    memset(&a, 0, sizeof(a));
    a.q = q;
    a.k_new = k;
    a.v_new = v;
    a.kc = k_cache;
    a.vc = v_cache;
    a.head_stride = (long long)max_seq * head_dim;
    a.seq_stride = a.head_stride * n_kv_heads;
    a.sin_tab = rope_sin;
    a.cos_tab = rope_cos;
    a.H = n_heads;
    a.HK = n_kv_heads;
    a.half = half;
    a.n_q = 1;
    a.q_pos0 = (long long)pos;
    a.rope = 1;
    a.vec = half % 4 == 0 && ((uintptr_t)rope_sin | (uintptr_t)rope_cos) % 16 == 0;
    a.append = 1;
    a.append_idx = (long long)pos;
    a.hist_len0 = hist;
    a.hist_step = 0;
    a.n_splits = n_splits;
    a.l2_ahead = kDefaultL2Ahead;
    a.chunk = hist > 0 ? (hist + n_splits - 1) / n_splits : 1;
    a.scale = 1.0f / sqrtf((float)head_dim);
    a.out_mode = 0;
    a.ao = ao;
    a.ws_m = ws_m;
    a.ws_l = ws_l;
    a.ws_acc = ws_acc;
    a.err = err_flag;
    void* params[] = {&a};
    dim3 grid((unsigned)n_splits, (unsigned)n_kv_heads, (unsigned)n_seqs);
    e = cudaLaunchKernel(kern.fn, grid, dim3(kern.threads), params, kern.smem, st);
    if (e != cudaSuccess) { report("cudaLaunchKernel", e); return PICKLE_ERR_DEVICE; }
    if (n_splits > 1) {
        MergeArgs m;
        memset(&m, 0, sizeof(m));
        m.ws_m = ws_m;
        m.ws_l = ws_l;
        m.ws_acc = ws_acc;
        m.n_splits = n_splits;
        m.out_mode = 0;
        m.out = ao;
        e = launch_decode_merge(head_dim, m, n_seqs * n_heads, st);
        if (e != cudaSuccess) { report("merge launch", e); return PICKLE_ERR_DEVICE; }
    }
    return PICKLE_OK;
}
