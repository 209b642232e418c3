// pickle_cuda.cu - the C ABI of include/pickle_cuda.h: handle, device KV
// cache, RoPE tables, launch planning and the host-buffer entry points that
// pickle's forward pass calls in place of its OpenMP attention block
// (lee-muriithi-kingori/lestramanika src/pickle_fast.c:1910-2109).
#include "pickle_cuda.h"

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "decode_splitkv.cuh"
#include "decode_xchg.cuh"
#include "prefill_common.cuh"
#include "prefill_tc.cuh"
#include "xchg_internal.cuh"

namespace {

struct KernelInfo {
    const void* fn = nullptr;
    int threads = 0;
    size_t smem = 0;
    int tile_rows = 32;
    int occupancy = 0;        // resident CTAs per SM, queried at first use
};

struct pickle_cuda_impl;

}  // namespace

struct pickle_cuda {
    int n_layers, H, HK, D, G, half, max_seq, n_seqs, rope_len, device, num_sms;
    int l2_ahead = kDefaultL2Ahead;   // decode tiles kept requested into L2 ahead of the ring
    int early_l2 = 2;         // decode tiles requested into L2 before the dependent-launch wait (measured best of 0, 2, 3, 4, 6)
    int pdl = 1;              // split kernel launched as a programmatic dependent of the kernel before it
    int force_splits = 0;     // > 0: split count for every decode (tuning sweeps), else planned
    size_t head_stride, seq_stride, layer_stride;   // floats
    float* kc = nullptr;
    float* vc = nullptr;
    float* sin_tab = nullptr;
    float* cos_tab = nullptr;
    float* ws_m = nullptr;
    float* ws_l = nullptr;
    float* ws_acc = nullptr;
    size_t ws_rows = 0;        // capacity in (group * G * split) rows
    int* err_dev = nullptr;
    unsigned* prefill_next = nullptr;   // next-item counter of the persistent prefill, zero between launches
    cudaStream_t stream = nullptr;
    // Host-buffer entry points: pinned staging and its device mirror.
    float* stage_host = nullptr;
    float* stage_dev = nullptr;
    size_t stage_cap = 0;      // floats
    // Prefill scratch: rotated q (F32) and BF16 operand copies.
    void* scratch = nullptr;
    size_t scratch_cap = 0;    // bytes
    KernelInfo decode;
    char last_error[256] = {0};
};

namespace {

int fail(pickle_cuda* h, cudaError_t e, const char* what) {
    if (h) snprintf(h->last_error, sizeof(h->last_error), "%s: %s", what, cudaGetErrorString(e));
    return PICKLE_ERR_DEVICE;
}

#define PCU_CHECK(h, call)                                            \
    do {                                                              \
        cudaError_t e_ = (call);                                      \
        if (e_ != cudaSuccess) return fail((h), e_, #call);           \
    } while (0)

template <int D, int G>
KernelInfo make_decode_info() {
    using C = DecodeCfg<D, G>;
    KernelInfo k;
    k.fn = reinterpret_cast<const void*>(&decode_splitkv_kernel<D, G>);
    k.threads = C::THREADS;
    k.smem = C::SMEM;
    k.tile_rows = C::TP;
    return k;
}

template <int D>
bool decode_info_for_g(int G, KernelInfo* out) {
    switch (G) {
        case 1: *out = make_decode_info<D, 1>(); return true;
        case 2: *out = make_decode_info<D, 2>(); return true;
        case 4: *out = make_decode_info<D, 4>(); return true;
        case 8: *out = make_decode_info<D, 8>(); return true;
        default: return false;
    }
}

// Head dims and GQA group sizes with a compiled decode kernel.
bool decode_info(int D, int G, KernelInfo* out) {
    switch (D) {
        case 48: return decode_info_for_g<48>(G, out);
        case 64: return decode_info_for_g<64>(G, out);
        case 96: return decode_info_for_g<96>(G, out);
        case 128: return decode_info_for_g<128>(G, out);
        case 256: return decode_info_for_g<256>(G, out);
        default: return false;
    }
}

int prepare_kernel(pickle_cuda* h, KernelInfo& k) {
    if (k.occupancy > 0) return PICKLE_OK;
    PCU_CHECK(h, cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)k.smem));
    int occ = 0;
    PCU_CHECK(h, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k.fn, k.threads, k.smem));
    if (occ < 1) {
        snprintf(h->last_error, sizeof(h->last_error), "decode kernel does not fit on an SM");
        return PICKLE_ERR_DEVICE;
    }
    k.occupancy = occ;
    return PICKLE_OK;
}

// Pick the number of KV splits for `groups` independent (seq, kv_head)
// streams of `hist` rows (the cost model of plan_decode_splits), with at
// least two tiles a split and no more partial rows than the workspace holds.
int plan_splits(const pickle_cuda* h, long long groups, long long hist) {
    const long long slots = (long long)h->num_sms * h->decode.occupancy;
    const long long tile = h->decode.tile_rows;
    long long max_s = hist / (2 * tile);
    if (max_s < 1) max_s = 1;
    if (max_s > kMaxSplits) max_s = kMaxSplits;
    const long long cap = (long long)(h->ws_rows / (size_t)h->G) / (groups > 0 ? groups : 1);
    if (max_s > cap) max_s = cap;
    if (max_s < 1) max_s = 1;
    if (h->force_splits > 0) {
        const long long s = h->force_splits < max_s ? h->force_splits : max_s;
        const long long chunk = (hist + s - 1) / s;
        return (int)((hist + chunk - 1) / chunk);
    }
    return plan_decode_splits(groups, hist, slots, max_s, h->G, h->D);
}

int check_layer(pickle_cuda* h, int layer, int n_seqs) {
    if (!h || layer < 0 || layer >= h->n_layers || n_seqs < 1 || n_seqs > h->n_seqs) return PICKLE_ERR_ARG;
    return PICKLE_OK;
}

DecodeArgs base_args(pickle_cuda* h, int layer) {
    DecodeArgs a;
    memset(&a, 0, sizeof(a));
    a.kc = h->kc + (size_t)layer * h->layer_stride;
    a.vc = h->vc + (size_t)layer * h->layer_stride;
    a.seq_stride = (long long)h->seq_stride;
    a.head_stride = (long long)h->head_stride;
    a.sin_tab = h->sin_tab;
    a.cos_tab = h->cos_tab;
    a.H = h->H;
    a.HK = h->HK;
    a.half = h->half;
    a.vec = h->half % 4 == 0;                 // table rows then start on 16-byte boundaries
    a.n_q = 1;
    a.l2_ahead = h->l2_ahead;
    a.early_l2 = h->early_l2;
    a.scale = 1.0f / sqrtf((float)h->D);      // src/pickle_fast.c:1959
    a.ws_m = h->ws_m;
    a.ws_l = h->ws_l;
    a.ws_acc = h->ws_acc;
    a.err = h->err_dev;
    return a;
}

int launch_decode(pickle_cuda* h, DecodeArgs& a, int n_z, cudaStream_t st) {
    int rc = prepare_kernel(h, h->decode);
    if (rc != PICKLE_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.n_splits, (unsigned)h->HK, (unsigned)n_z);
    cfg.blockDim = dim3(h->decode.threads);
    cfg.dynamicSmemBytes = h->decode.smem;
    cfg.stream = st;
    // The kernel waits for the kernel before it (griddepcontrol.wait) before
    // its first global access, so its CTAs may become resident early.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = h->pdl ? 1 : 0;
    void* params[] = {&a};
    PCU_CHECK(h, cudaLaunchKernelExC(&cfg, h->decode.fn, params));
    if (a.n_splits > 1) {
        MergeArgs m;
        memset(&m, 0, sizeof(m));
        m.ws_m = a.ws_m;
        m.ws_l = a.ws_l;
        m.ws_acc = a.ws_acc;
        m.n_splits = a.n_splits;
        m.out_mode = a.out_mode;
        m.out = a.ao;
        m.out_m = a.out_m;
        m.out_l = a.out_l;
        PCU_CHECK(h, launch_decode_merge(h->D, m, n_z * h->H, st));   // one row per (query, head)
    }
    return PICKLE_OK;
}

// Arguments of the split kernel for n_seqs queries at `pos` over `hist`
// cached rows, optionally appending the new row at `append_idx`.
int decode_args(pickle_cuda* h, int layer, int n_seqs, size_t pos, long long hist, int append,
                long long append_idx, const float* q, const float* k, const float* v, float* ao,
                float* m_out, float* l_out, int out_mode, DecodeArgs* out) {
    int rc = prepare_kernel(h, h->decode);
    if (rc != PICKLE_OK) return rc;
    const long long groups = (long long)n_seqs * h->HK;
    // Query, new rows and outputs move as 16-byte vectors.
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)ao) % 16) {
        snprintf(h->last_error, sizeof(h->last_error), "q, k, v and output rows must be 16-byte aligned");
        return PICKLE_ERR_ARG;
    }
    DecodeArgs& a = *out;
    a = base_args(h, layer);
    a.q = q;
    a.k_new = k;
    a.v_new = v;
    a.q_pos0 = (long long)pos;
    a.rope = 1;
    a.append = append;
    a.append_idx = append_idx;
    a.hist_len0 = hist;
    a.hist_step = 0;
    a.n_splits = hist > 0 ? plan_splits(h, groups, hist) : 1;
    a.chunk = hist > 0 ? (hist + a.n_splits - 1) / a.n_splits : 1;
    a.out_mode = out_mode;
    a.ao = ao;
    a.out_m = m_out;
    a.out_l = l_out;
    return PICKLE_OK;
}

// Decode of n_seqs queries: the split kernel and, with several splits, the merge.
int decode_common(pickle_cuda* h, int layer, int n_seqs, size_t pos, long long hist, int append,
                  long long append_idx, const float* q, const float* k, const float* v, float* ao,
                  float* m_out, float* l_out, int out_mode, cudaStream_t st) {
    DecodeArgs a;
    int rc = decode_args(h, layer, n_seqs, pos, hist, append, append_idx, q, k, v, ao, m_out, l_out, out_mode, &a);
    if (rc != PICKLE_OK) return rc;
    return launch_decode(h, a, n_seqs, st);
}

// An exchange every rank of which is reachable, on the handle's device.
int check_xchg(pickle_cuda* h, pickle_cuda_xchg* x) {
    if (!x) return PICKLE_ERR_ARG;
    if (x->device != h->device) {
        snprintf(h->last_error, sizeof(h->last_error), "exchange on device %d, handle on device %d", x->device,
                 h->device);
        return PICKLE_ERR_ARG;
    }
    if (x->broken) {
        snprintf(h->last_error, sizeof(h->last_error), "exchange broken by an earlier wait that gave up: recreate it");
        return PICKLE_ERR_DEVICE;
    }
    for (int p = 0; p < x->world; ++p)
        if (!x->opened[p]) {
            snprintf(h->last_error, sizeof(h->last_error), "peer %d's region is not open", p);
            return PICKLE_ERR_ARG;
        }
    return PICKLE_OK;
}

// The split kernel writing partials (one split included), then the fused
// merge + exchange as its programmatic dependent.
int launch_decode_xchg(pickle_cuda* h, pickle_cuda_xchg* x, DecodeArgs& a, int n_z, XchgMergeArgs& xm,
                       cudaStream_t st) {
    a.force_partials = 1;
    // As in launch_decode: the split kernel is a programmatic dependent of
    // the kernel before it (the previous step's merge-exchange launch, which
    // triggers at its start), so its CTAs become resident while that one ends.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.n_splits, (unsigned)h->HK, (unsigned)n_z);
    cfg.blockDim = dim3(h->decode.threads);
    cfg.dynamicSmemBytes = h->decode.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = h->pdl ? 1 : 0;
    void* params[] = {&a};
    PCU_CHECK(h, cudaLaunchKernelExC(&cfg, h->decode.fn, params));
    memset(&xm.m, 0, sizeof(xm.m));
    xm.m.ws_m = a.ws_m;
    xm.m.ws_l = a.ws_l;
    xm.m.ws_acc = a.ws_acc;
    xm.m.n_splits = a.n_splits;
    xm.px = xchg_peers(x);
    xm.n_rows = n_z * h->H;
    xm.err = x->err_dev;
    PCU_CHECK(h, launch_decode_merge_xchg(h->D, xm, st));
    return PICKLE_OK;
}

int ensure_stage(pickle_cuda* h, size_t floats) {
    if (floats <= h->stage_cap) return PICKLE_OK;
    if (h->stage_host) cudaFreeHost(h->stage_host);
    if (h->stage_dev) cudaFree(h->stage_dev);
    h->stage_host = nullptr;
    h->stage_dev = nullptr;
    h->stage_cap = 0;
    PCU_CHECK(h, cudaMallocHost(&h->stage_host, floats * sizeof(float)));
    PCU_CHECK(h, cudaMalloc(&h->stage_dev, floats * sizeof(float)));
    h->stage_cap = floats;
    return PICKLE_OK;
}

int ensure_scratch(pickle_cuda* h, size_t bytes) {
    if (bytes <= h->scratch_cap) return PICKLE_OK;
    if (h->scratch) cudaFree(h->scratch);
    h->scratch = nullptr;
    h->scratch_cap = 0;
    PCU_CHECK(h, cudaMalloc(&h->scratch, bytes));
    h->scratch_cap = bytes;
    return PICKLE_OK;
}

// Read and clear the device error word; PICKLE_ERR_DEVICE if it was set.
int take_device_error(pickle_cuda* h, cudaStream_t st) {
    int err = 0;
    PCU_CHECK(h, cudaMemcpyAsync(&err, h->err_dev, sizeof(int), cudaMemcpyDeviceToHost, st));
    PCU_CHECK(h, cudaStreamSynchronize(st));
    if (err != 0) {
        snprintf(h->last_error, sizeof(h->last_error), "device wait gave up (code %d)", err);
        PCU_CHECK(h, cudaMemsetAsync(h->err_dev, 0, sizeof(int), st));
        // A launch that gave up may leave the persistent prefill's item counter part-way.
        PCU_CHECK(h, cudaMemsetAsync(h->prefill_next, 0, sizeof(unsigned), st));
        PCU_CHECK(h, cudaStreamSynchronize(st));
        return PICKLE_ERR_DEVICE;
    }
    return PICKLE_OK;
}

int prefill_launch(pickle_cuda* h, int layer, int n_seqs, size_t pos0, size_t T, const float* q,
                   const float* k, const float* v, float* ao, int precision, cudaStream_t st, int slot0 = 0);

}  // namespace

extern "C" {

int pickle_cuda_abi_version(void) { return PICKLE_CUDA_ABI_VERSION; }

int pickle_cuda_init(const pickle_cuda_params_t* p, int device, pickle_cuda_t** out) {
    if (!p || !out) return PICKLE_ERR_ARG;
    *out = nullptr;
    if (p->n_layers <= 0 || p->n_heads <= 0 || p->n_kv_heads <= 0 || p->head_dim <= 0 ||
        p->max_seq <= 0 || p->n_seqs <= 0 || p->n_heads % p->n_kv_heads != 0 ||
        p->head_dim % 4 != 0 || p->half < 0 || 2 * p->half > p->head_dim || p->rope_len < 0)
        return PICKLE_ERR_ARG;
    KernelInfo info;
    if (!decode_info(p->head_dim, p->n_heads / p->n_kv_heads, &info)) return PICKLE_ERR_ARG;

    pickle_cuda* h = new (std::nothrow) pickle_cuda();
    if (!h) return PICKLE_ERR_MEMORY;
    h->n_layers = p->n_layers;
    h->H = p->n_heads;
    h->HK = p->n_kv_heads;
    h->D = p->head_dim;
    h->G = p->n_heads / p->n_kv_heads;
    h->half = p->half;
    h->max_seq = p->max_seq;
    h->n_seqs = p->n_seqs;
    h->rope_len = p->rope_len > 0 ? p->rope_len : p->max_seq;
    h->device = device;
    h->decode = info;
    // Tuning knob for sweeps of the L2 look-ahead (tiles, 0 turns it off).
    if (const char* env = getenv("PICKLE_CUDA_L2_AHEAD")) {
        const int v = atoi(env);
        if (v >= 0 && v <= 64) h->l2_ahead = v;
    }
    if (const char* env = getenv("PICKLE_CUDA_EARLY_L2")) {
        const int v = atoi(env);
        if (v >= 0 && v <= 64) h->early_l2 = v;
    }
    // Knob for A/B timing of the dependent launch (0 turns it off).
    if (const char* env = getenv("PICKLE_CUDA_PDL")) h->pdl = atoi(env) != 0;
    // Knob for split-count sweeps (the planner's choice when unset).
    if (const char* env = getenv("PICKLE_CUDA_SPLITS")) h->force_splits = atoi(env);
    h->head_stride = (size_t)p->max_seq * p->head_dim;
    h->seq_stride = h->head_stride * p->n_kv_heads;
    h->layer_stride = h->seq_stride * p->n_seqs;

    auto bail = [&](int rc) { pickle_cuda_free(h); return rc; };
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) { fail(h, e, "cudaSetDevice"); return bail(PICKLE_ERR_DEVICE); }
    e = cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) { fail(h, e, "cudaDeviceGetAttribute"); return bail(PICKLE_ERR_DEVICE); }
    e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) { fail(h, e, "cudaStreamCreate"); return bail(PICKLE_ERR_DEVICE); }

    const size_t cache_bytes = h->layer_stride * (size_t)h->n_layers * sizeof(float);
    if (cudaMalloc(&h->kc, cache_bytes) != cudaSuccess || cudaMalloc(&h->vc, cache_bytes) != cudaSuccess)
        return bail(PICKLE_ERR_MEMORY);
    if (cudaMemset(h->kc, 0, cache_bytes) != cudaSuccess || cudaMemset(h->vc, 0, cache_bytes) != cudaSuccess)
        return bail(PICKLE_ERR_DEVICE);

    // RoPE tables on the host with the host's libm, exactly as
    // pickle_fast_state_extend_rope fills them (src/pickle_fast.c:1772-1788).
    const int half = h->half;
    const size_t tab = (size_t)h->rope_len * (half > 0 ? half : 1);
    float* inv = (float*)calloc((size_t)(half > 0 ? half : 1), sizeof(float));
    float* hs = (float*)malloc(tab * sizeof(float));
    float* hc = (float*)malloc(tab * sizeof(float));
    if (!inv || !hs || !hc) { free(inv); free(hs); free(hc); return bail(PICKLE_ERR_MEMORY); }
    for (int i = 0; i < half; ++i)
        inv[i] = p->rope_inv_freq ? p->rope_inv_freq[i]
                                  : 1.0f / powf(p->rope_theta, (float)(2 * i) / (float)p->head_dim);
    for (int pos = 0; pos < h->rope_len; ++pos)
        for (int i = 0; i < half; ++i) {
            const float angle = inv[i] * (float)pos;
            hs[(size_t)pos * half + i] = sinf(angle);
            hc[(size_t)pos * half + i] = cosf(angle);
        }
    bool ok = cudaMalloc(&h->sin_tab, tab * sizeof(float)) == cudaSuccess &&
              cudaMalloc(&h->cos_tab, tab * sizeof(float)) == cudaSuccess &&
              cudaMemcpy(h->sin_tab, hs, tab * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(h->cos_tab, hc, tab * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess;
    free(inv); free(hs); free(hc);
    if (!ok) return bail(PICKLE_ERR_DEVICE);

    // Split-KV workspace: at most 4096 partial rows per KV group member.
    h->ws_rows = (size_t)4096 * h->G;
    ok = cudaMalloc(&h->ws_m, h->ws_rows * sizeof(float)) == cudaSuccess &&
         cudaMalloc(&h->ws_l, h->ws_rows * sizeof(float)) == cudaSuccess &&
         cudaMalloc(&h->ws_acc, h->ws_rows * h->D * sizeof(float)) == cudaSuccess &&
         cudaMalloc(&h->err_dev, sizeof(int)) == cudaSuccess &&
         cudaMalloc(&h->prefill_next, sizeof(unsigned)) == cudaSuccess &&
         cudaMemset(h->prefill_next, 0, sizeof(unsigned)) == cudaSuccess &&
         cudaMemset(h->err_dev, 0, sizeof(int)) == cudaSuccess;
    if (!ok) return bail(PICKLE_ERR_MEMORY);
    if (prepare_kernel(h, h->decode) != PICKLE_OK) return bail(PICKLE_ERR_DEVICE);
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(PICKLE_ERR_DEVICE);
    *out = h;
    return PICKLE_OK;
}

void pickle_cuda_free(pickle_cuda_t* h) {
    if (!h) return;
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    cudaFree(h->kc); cudaFree(h->vc);
    cudaFree(h->sin_tab); cudaFree(h->cos_tab);
    cudaFree(h->ws_m); cudaFree(h->ws_l); cudaFree(h->ws_acc);
    cudaFree(h->err_dev);
    cudaFree(h->prefill_next);
    cudaFree(h->stage_dev); cudaFree(h->scratch);
    if (h->stage_host) cudaFreeHost(h->stage_host);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

const char* pickle_cuda_last_error(pickle_cuda_t* h) { return h ? h->last_error : "null handle"; }

int pickle_cuda_decode_plan(pickle_cuda_t* h, int n_seqs, size_t pos, int* n_splits, int* n_launches) {
    if (!h || n_seqs < 1) return PICKLE_ERR_ARG;
    int rc = prepare_kernel(h, h->decode);
    if (rc != PICKLE_OK) return rc;
    const long long hist = (long long)pos;
    const int s = hist > 0 ? plan_splits(h, (long long)n_seqs * h->HK, hist) : 1;
    if (n_splits) *n_splits = s;
    if (n_launches) *n_launches = s > 1 ? 2 : 1;    // split kernel (+ merge kernel)
    return PICKLE_OK;
}

int pickle_cuda_decode_batch_dev(pickle_cuda_t* h, int layer, int n_seqs, size_t pos, const float* q,
                                 const float* k, const float* v, float* ao, void* stream) {
    int rc = check_layer(h, layer, n_seqs);
    if (rc != PICKLE_OK) return rc;
    if (pos >= (size_t)h->max_seq || pos >= (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    if (!q || !k || !v || !ao) return PICKLE_ERR_ARG;
    return decode_common(h, layer, n_seqs, pos, (long long)pos, 1, (long long)pos, q, k, v, ao,
                         nullptr, nullptr, 0, (cudaStream_t)stream);
}

int pickle_cuda_decode_ragged_dev(pickle_cuda_t* h, int layer, int n, const int* pos_dev, const int* slot_dev,
                                  size_t max_pos, const float* q, const float* k, const float* v, float* ao,
                                  void* stream) {
    int rc = check_layer(h, layer, n);
    if (rc != PICKLE_OK) return rc;
    if (!pos_dev || !q || !k || !v || !ao) return PICKLE_ERR_ARG;
    if (max_pos >= (size_t)h->max_seq || max_pos >= (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    rc = prepare_kernel(h, h->decode);
    if (rc != PICKLE_OK) return rc;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)ao) % 16) {
        snprintf(h->last_error, sizeof(h->last_error), "q, k, v and output rows must be 16-byte aligned");
        return PICKLE_ERR_ARG;
    }
    // Splits are planned for the longest entry; each entry cuts its own
    // history into that many pieces on the device.
    DecodeArgs a = base_args(h, layer);
    a.q = q;
    a.k_new = k;
    a.v_new = v;
    a.rope = 1;
    a.append = 1;
    a.n_splits = max_pos > 0 ? plan_splits(h, (long long)n * h->HK, (long long)max_pos) : 1;
    a.out_mode = 0;
    a.ao = ao;
    a.seq_pos = pos_dev;
    a.seq_slot = slot_dev;
    a.max_pos = (long long)max_pos;
    a.n_slots = h->n_seqs;
    return launch_decode(h, a, n, (cudaStream_t)stream);
}

int pickle_cuda_decode_partial_dev(pickle_cuda_t* h, int layer, int n_seqs, size_t pos, size_t n_local,
                                   int append, const float* q, const float* k, const float* v,
                                   float* m_out, float* l_out, float* acc_out, void* stream) {
    int rc = check_layer(h, layer, n_seqs);
    if (rc != PICKLE_OK) return rc;
    if (!q || !m_out || !l_out || !acc_out || (append && (!k || !v))) return PICKLE_ERR_ARG;
    if (n_local + (append ? 1 : 0) > (size_t)h->max_seq) return PICKLE_ERR_RANGE;
    if (n_local == 0 && !append) return PICKLE_ERR_ARG;
    if (pos >= (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    return decode_common(h, layer, n_seqs, pos, (long long)n_local, append ? 1 : 0, (long long)n_local,
                         q, k, v, acc_out, m_out, l_out, 1, (cudaStream_t)stream);
}

int pickle_cuda_decode_gather_dev(pickle_cuda_t* h, pickle_cuda_xchg_t* x, int layer, int n_seqs, size_t pos,
                                  const float* q, const float* k, const float* v, float* out, void* stream) {
    int rc = check_layer(h, layer, n_seqs);
    if (rc != PICKLE_OK) return rc;
    if (!q || !k || !v || !out) return PICKLE_ERR_ARG;
    if ((uintptr_t)out % 16) return PICKLE_ERR_ARG;
    if (pos >= (size_t)h->max_seq || pos >= (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    rc = check_xchg(h, x);
    if (rc != PICKLE_OK) return rc;
    const int n_rows = n_seqs * h->H;
    if (n_rows > kXchgMaxRows || decode_xchg_bytes(0, x->world, n_rows, h->D) > x->buf_bytes)
        return PICKLE_ERR_RANGE;
    DecodeArgs a;
    // ao is unused: the partials go to the workspace; `out` passes the alignment check.
    rc = decode_args(h, layer, n_seqs, pos, (long long)pos, 1, (long long)pos, q, k, v, out, nullptr, nullptr, 0,
                     &a);
    if (rc != PICKLE_OK) return rc;
    XchgMergeArgs xm;
    memset(&xm, 0, sizeof(xm));
    xm.mode = 0;
    xm.rows_per_z = h->H;
    xm.row_bytes = (unsigned long long)h->D * 8;
    xm.out = out;
    return launch_decode_xchg(h, x, a, n_seqs, xm, (cudaStream_t)stream);
}

int pickle_cuda_decode_seqshard_dev(pickle_cuda_t* h, pickle_cuda_xchg_t* x, int layer, int n_seqs, size_t pos,
                                    size_t n_local, int append, const float* q, const float* k, const float* v,
                                    float* out, void* stream) {
    int rc = check_layer(h, layer, n_seqs);
    if (rc != PICKLE_OK) return rc;
    if (!q || !out || (append && (!k || !v))) return PICKLE_ERR_ARG;
    if (n_local + (append ? 1 : 0) > (size_t)h->max_seq) return PICKLE_ERR_RANGE;
    if (n_local == 0 && !append) return PICKLE_ERR_ARG;
    if (pos >= (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    rc = check_xchg(h, x);
    if (rc != PICKLE_OK) return rc;
    const int n_rows = n_seqs * h->H;
    if (n_rows > kXchgMaxRows || decode_xchg_bytes(1, x->world, n_rows, h->D) > x->buf_bytes)
        return PICKLE_ERR_RANGE;
    DecodeArgs a;
    rc = decode_args(h, layer, n_seqs, pos, (long long)n_local, append ? 1 : 0, (long long)n_local, q, k, v, out,
                     nullptr, nullptr, 1, &a);
    if (rc != PICKLE_OK) return rc;
    XchgMergeArgs xm;
    memset(&xm, 0, sizeof(xm));
    xm.mode = 1;
    xm.row_bytes = (unsigned long long)(h->D + 2) * 8;
    xm.out = out;
    return launch_decode_xchg(h, x, a, n_seqs, xm, (cudaStream_t)stream);
}

int pickle_cuda_decode_xchg_bytes(int sharding, int world, int n_seqs, int n_heads, int head_dim, size_t* bytes) {
    if ((sharding != PICKLE_CUDA_SHARD_HEADS && sharding != PICKLE_CUDA_SHARD_SEQ) || world < 1 ||
        world > kXchgMaxRanks || n_seqs < 1 || n_heads < 1 || head_dim < 4 || head_dim % 4 || !bytes)
        return PICKLE_ERR_ARG;
    if ((size_t)n_seqs * n_heads > (size_t)kXchgMaxRows) return PICKLE_ERR_RANGE;
    *bytes = decode_xchg_bytes(sharding == PICKLE_CUDA_SHARD_HEADS ? 0 : 1, world, n_seqs * n_heads, head_dim);
    return PICKLE_OK;
}

int pickle_cuda_lse_merge_dev(int n_parts, int n_rows, int head_dim, const float* m_in, const float* l_in,
                              const float* acc_in, float* out, void* stream) {
    if (n_parts < 1 || n_rows < 1 || head_dim < 1 || !m_in || !l_in || !acc_in || !out) return PICKLE_ERR_ARG;
    lse_merge_kernel<<<n_rows, head_dim < 128 ? 64 : 128, 0, (cudaStream_t)stream>>>(
        n_parts, n_rows, head_dim, n_rows, (long long)n_rows * head_dim, m_in, l_in, acc_in, out);
    return cudaGetLastError() == cudaSuccess ? PICKLE_OK : PICKLE_ERR_DEVICE;
}

int pickle_cuda_lse_merge_packed_dev(int n_parts, int n_rows, int head_dim, const float* parts,
                                     size_t part_stride, float* out, void* stream) {
    if (n_parts < 1 || n_rows < 1 || head_dim < 1 || !parts || !out ||
        part_stride < (size_t)n_rows * (head_dim + 2))
        return PICKLE_ERR_ARG;
    const float* acc = parts;
    const float* m = parts + (size_t)n_rows * head_dim;
    const float* l = m + n_rows;
    lse_merge_kernel<<<n_rows, head_dim < 128 ? 64 : 128, 0, (cudaStream_t)stream>>>(
        n_parts, n_rows, head_dim, (long long)part_stride, (long long)part_stride, m, l, acc, out);
    return cudaGetLastError() == cudaSuccess ? PICKLE_OK : PICKLE_ERR_DEVICE;
}

int pickle_cuda_attn_decode(pickle_cuda_t* h, int layer, size_t pos, const float* q, const float* k,
                            const float* v, float* ao) {
    int rc = check_layer(h, layer, 1);
    if (rc != PICKLE_OK) return rc;
    if (!q || !k || !v || !ao) return PICKLE_ERR_ARG;
    if (pos >= (size_t)h->max_seq || pos >= (size_t)h->rope_len) return PICKLE_ERR_RANGE;  // src/pickle_fast.c:1885
    const size_t nq = (size_t)h->H * h->D, nk = (size_t)h->HK * h->D;
    rc = ensure_stage(h, 2 * nq + 2 * nk);
    if (rc != PICKLE_OK) return rc;
    PCU_CHECK(h, cudaSetDevice(h->device));
    float* hs = h->stage_host;
    memcpy(hs, q, nq * sizeof(float));
    memcpy(hs + nq, k, nk * sizeof(float));
    memcpy(hs + nq + nk, v, nk * sizeof(float));
    float* ds = h->stage_dev;
    PCU_CHECK(h, cudaMemcpyAsync(ds, hs, (nq + 2 * nk) * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    float* dao = ds + nq + 2 * nk;
    rc = decode_common(h, layer, 1, pos, (long long)pos, 1, (long long)pos, ds, ds + nq, ds + nq + nk,
                       dao, nullptr, nullptr, 0, h->stream);
    if (rc != PICKLE_OK) return rc;
    PCU_CHECK(h, cudaMemcpyAsync(hs + nq + 2 * nk, dao, nq * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    rc = take_device_error(h, h->stream);
    if (rc != PICKLE_OK) return rc;
    memcpy(ao, hs + nq + 2 * nk, nq * sizeof(float));
    return PICKLE_OK;
}

int pickle_cuda_prefill_dev(pickle_cuda_t* h, int layer, int n_seqs, size_t pos0, size_t T, const float* q,
                            const float* k, const float* v, float* ao, int precision, void* stream) {
    int rc = check_layer(h, layer, n_seqs);
    if (rc != PICKLE_OK) return rc;
    if (!q || !k || !v || !ao || T == 0) return PICKLE_ERR_ARG;
    if (pos0 + T > (size_t)h->max_seq || pos0 + T > (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    if (precision != PICKLE_CUDA_PREFILL_F32 && precision != PICKLE_CUDA_PREFILL_BF16) return PICKLE_ERR_ARG;
    return prefill_launch(h, layer, n_seqs, pos0, T, q, k, v, ao, precision, (cudaStream_t)stream);
}

int pickle_cuda_prefill_slot_dev(pickle_cuda_t* h, int layer, int slot, size_t pos0, size_t T, const float* q,
                                 const float* k, const float* v, float* ao, int precision, void* stream) {
    int rc = check_layer(h, layer, 1);
    if (rc != PICKLE_OK) return rc;
    if (slot < 0 || slot >= h->n_seqs) return PICKLE_ERR_RANGE;
    if (!q || !k || !v || !ao || T == 0) return PICKLE_ERR_ARG;
    if (pos0 + T > (size_t)h->max_seq || pos0 + T > (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    if (precision != PICKLE_CUDA_PREFILL_F32 && precision != PICKLE_CUDA_PREFILL_BF16) return PICKLE_ERR_ARG;
    return prefill_launch(h, layer, 1, pos0, T, q, k, v, ao, precision, (cudaStream_t)stream, slot);
}

int pickle_cuda_prefill_attn_bf16_dev(int n_seqs, int T, int n_heads, int n_kv_heads, int head_dim,
                                      const void* q_bf16, const void* k_bf16, const void* v_bf16, float* ao,
                                      int* err_flag, void* stream) {
    if (n_seqs < 1 || T < 1 || n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads || !q_bf16 || !k_bf16 ||
        !v_bf16 || !ao)
        return PICKLE_ERR_ARG;
    if (!prefill_tc_supported(head_dim, n_heads / n_kv_heads)) return PICKLE_ERR_ARG;
    char msg[256];
    int rc = prefill_tc_launch((const __nv_bfloat16*)q_bf16, (const __nv_bfloat16*)k_bf16,
                               (const __nv_bfloat16*)v_bf16, ao, n_seqs, T, n_heads, n_kv_heads, head_dim,
                               1.0f / sqrtf((float)head_dim), err_flag, nullptr, (cudaStream_t)stream, msg,
                               sizeof(msg));
    if (rc != 0) fprintf(stderr, "pickle_cuda_prefill_attn_bf16_dev: %s\n", msg);
    return rc == 0 ? PICKLE_OK : (rc == -6 ? PICKLE_ERR_ARG : PICKLE_ERR_DEVICE);
}

int pickle_cuda_attn_prefill(pickle_cuda_t* h, int layer, size_t pos0, size_t T, const float* q,
                             const float* k, const float* v, float* ao, int precision) {
    int rc = check_layer(h, layer, 1);
    if (rc != PICKLE_OK) return rc;
    if (!q || !k || !v || !ao || T == 0) return PICKLE_ERR_ARG;
    if (pos0 + T > (size_t)h->max_seq || pos0 + T > (size_t)h->rope_len) return PICKLE_ERR_RANGE;
    const size_t nq = T * h->H * h->D, nk = T * h->HK * h->D;
    rc = ensure_stage(h, 2 * nq + 2 * nk);
    if (rc != PICKLE_OK) return rc;
    PCU_CHECK(h, cudaSetDevice(h->device));
    float* hs = h->stage_host;
    memcpy(hs, q, nq * sizeof(float));
    memcpy(hs + nq, k, nk * sizeof(float));
    memcpy(hs + nq + nk, v, nk * sizeof(float));
    float* ds = h->stage_dev;
    PCU_CHECK(h, cudaMemcpyAsync(ds, hs, (nq + 2 * nk) * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    float* dao = ds + nq + 2 * nk;
    rc = pickle_cuda_prefill_dev(h, layer, 1, pos0, T, ds, ds + nq, ds + nq + nk, dao, precision, h->stream);
    if (rc != PICKLE_OK) return rc;
    PCU_CHECK(h, cudaMemcpyAsync(hs + nq + 2 * nk, dao, nq * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    rc = take_device_error(h, h->stream);
    if (rc != PICKLE_OK) return rc;
    memcpy(ao, hs + nq + 2 * nk, nq * sizeof(float));
    return PICKLE_OK;
}

int pickle_cuda_kv_write(pickle_cuda_t* h, int layer, int seq, size_t pos0, size_t n_pos, const float* k_host,
                         const float* v_host) {
    if (!h || layer < 0 || layer >= h->n_layers || seq < 0 || seq >= h->n_seqs || !k_host || !v_host)
        return PICKLE_ERR_ARG;
    if (pos0 + n_pos > (size_t)h->max_seq) return PICKLE_ERR_RANGE;
    if (n_pos == 0) return PICKLE_OK;
    PCU_CHECK(h, cudaSetDevice(h->device));
    const size_t row = (size_t)h->D * sizeof(float);
    for (int kvh = 0; kvh < h->HK; ++kvh) {
        const size_t off = (size_t)layer * h->layer_stride + (size_t)seq * h->seq_stride +
                           (size_t)kvh * h->head_stride + pos0 * h->D;
        PCU_CHECK(h, cudaMemcpy2DAsync(h->kc + off, row, k_host + (size_t)kvh * h->D, (size_t)h->HK * row, row,
                                       n_pos, cudaMemcpyHostToDevice, h->stream));
        PCU_CHECK(h, cudaMemcpy2DAsync(h->vc + off, row, v_host + (size_t)kvh * h->D, (size_t)h->HK * row, row,
                                       n_pos, cudaMemcpyHostToDevice, h->stream));
    }
    PCU_CHECK(h, cudaStreamSynchronize(h->stream));
    return PICKLE_OK;
}

int pickle_cuda_kv_layout(pickle_cuda_t* h, int layer, float** k_dev, float** v_dev, size_t* seq_stride,
                          size_t* head_stride) {
    if (!h || layer < 0 || layer >= h->n_layers) return PICKLE_ERR_ARG;
    if (k_dev) *k_dev = h->kc + (size_t)layer * h->layer_stride;
    if (v_dev) *v_dev = h->vc + (size_t)layer * h->layer_stride;
    if (seq_stride) *seq_stride = h->seq_stride;
    if (head_stride) *head_stride = h->head_stride;
    return PICKLE_OK;
}

int pickle_cuda_sync(pickle_cuda_t* h, void* stream) {
    if (!h) return PICKLE_ERR_ARG;
    PCU_CHECK(h, cudaSetDevice(h->device));
    PCU_CHECK(h, cudaGetLastError());
    return take_device_error(h, (cudaStream_t)stream);
}

}  // extern "C"

namespace {

// Vectorised producer when rows split into float4 rotation pairs, scalar otherwise.
void launch_rope_append(const RopeAppendArgs& ra, int T, int n_seqs, cudaStream_t st) {
    const bool vec = ra.D % 4 == 0 && ra.half % 4 == 0 &&
                     ((uintptr_t)ra.q | (uintptr_t)ra.k | (uintptr_t)ra.v) % 16 == 0;
    if (vec)
        rope_append_vec_kernel<<<dim3((unsigned)T, (unsigned)n_seqs), 128, 0, st>>>(ra);
    else
        rope_append_kernel<<<dim3((unsigned)T, (unsigned)n_seqs), 256, 0, st>>>(ra);
}

int prefill_launch(pickle_cuda* h, int layer, int n_seqs, size_t pos0, size_t T, const float* q,
                   const float* k, const float* v, float* ao, int precision, cudaStream_t st, int slot0) {
    const size_t nq = (size_t)n_seqs * T * h->H * h->D;
    const size_t nk = (size_t)n_seqs * T * h->HK * h->D;
    if ((uintptr_t)ao % 16) {
        snprintf(h->last_error, sizeof(h->last_error), "output rows must be 16-byte aligned");
        return PICKLE_ERR_ARG;
    }
    RopeAppendArgs ra;
    memset(&ra, 0, sizeof(ra));
    ra.q = q; ra.k = k; ra.v = v;
    // Sequences [slot0, slot0 + n_seqs) of the cache.
    ra.kc = h->kc + (size_t)layer * h->layer_stride + (size_t)slot0 * h->seq_stride;
    ra.vc = h->vc + (size_t)layer * h->layer_stride + (size_t)slot0 * h->seq_stride;
    ra.seq_stride = (long long)h->seq_stride;
    ra.head_stride = (long long)h->head_stride;
    ra.sin_tab = h->sin_tab; ra.cos_tab = h->cos_tab;
    ra.H = h->H; ra.HK = h->HK; ra.D = h->D; ra.half = h->half; ra.T = (int)T;
    ra.pos0 = (long long)pos0;
    ra.q_prescale = 1.0f;

    const bool tc = precision == PICKLE_CUDA_PREFILL_BF16 && prefill_tc_supported(h->D, h->H / h->HK) && pos0 == 0;
    if (!tc) {
        int rc = ensure_scratch(h, nq * sizeof(float));
        if (rc != PICKLE_OK) return rc;
        ra.q_rot = (float*)h->scratch;
        launch_rope_append(ra, (int)T, n_seqs, st);
        PCU_CHECK(h, cudaGetLastError());
        // Causal attention: query t of each sequence attends rows [0, pos0+t].
        DecodeArgs a = base_args(h, layer);
        a.kc = ra.kc;
        a.vc = ra.vc;
        a.q = (const float*)h->scratch;
        a.n_q = (int)T;
        a.q_pos0 = (long long)pos0;
        a.rope = 0;
        a.append = 0;
        a.hist_len0 = (long long)pos0 + 1;
        a.hist_step = 1;
        a.n_splits = 1;
        a.chunk = (long long)(pos0 + T);
        a.out_mode = 0;
        a.ao = ao;
        return launch_decode(h, a, (int)(n_seqs * T), st);
    }
    // Tensor-core path: BF16 head-major operand copies, then one causal launch.
    const size_t bq = nq * sizeof(__nv_bfloat16), bk = nk * sizeof(__nv_bfloat16);
    int rc = ensure_scratch(h, bq + 2 * bk + 1024);
    if (rc != PICKLE_OK) return rc;
    char* base = (char*)h->scratch;
    ra.q_bf16 = (__nv_bfloat16*)base;
    ra.k_bf16 = (__nv_bfloat16*)(base + bq);
    ra.v_bf16 = (__nv_bfloat16*)(base + bq + bk);
    launch_rope_append(ra, (int)T, n_seqs, st);
    PCU_CHECK(h, cudaGetLastError());
    return prefill_tc_launch(ra.q_bf16, ra.k_bf16, ra.v_bf16, ao, n_seqs, (int)T, h->H, h->HK, h->D,
                             1.0f / sqrtf((float)h->D), h->err_dev, h->prefill_next, st, h->last_error,
                             sizeof(h->last_error));
}

}  // namespace
