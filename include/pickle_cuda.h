/*
 * pickle_cuda.h - C ABI of the B200 attention block for pickle.
 *
 * This library replaces the per-layer GQA attention block of pickle's
 * host forward pass (lee-muriithi-kingori/lestramanika,
 * src/pickle_fast.c:1910-2109): RoPE (NeoX half-split) on q and k, the
 * KV-cache append, and causal softmax attention over positions [0, pos].
 * Around it: the weight projections (pickle_fast_matmul_dispatch, per
 * token and for whole prompts) and the whole forward pass with the greedy
 * decode loop (pickle_cuda_model_*, at the end of this header).
 *
 * Everything here is plain C: pointers, sizes and int status codes.
 * Status codes are pickle's own (src/pickle.h:52-60) plus
 * PICKLE_ERR_DEVICE for CUDA/NCCL failures.
 *
 * Ownership: host buffers (q, k, v, ao) belong to the caller. The device
 * KV cache, the RoPE sin/cos tables and the split-KV workspace belong to
 * the pickle_cuda_t handle. One handle is driven by one host thread and
 * one CUDA stream at a time (pickle_fast_forward is not re-entrant either,
 * src/pickle_fast.c:1857-1871 shares one set of work buffers).
 *
 * Device KV layout (head-major, 16-byte aligned rows):
 *     k[layer][seq][kv_head][max_seq][head_dim]   float32
 * replacing the host layout [layer][pos][kv_head][head_dim]
 * (src/pickle_fast.h:145-157). A contiguous run of positions of one
 * (layer, seq, kv_head) is one contiguous byte range, so a tile of keys
 * is a single bulk copy.
 */
#ifndef PICKLE_CUDA_H
#define PICKLE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: the first nine mirror src/pickle.h:52-60. */
#ifndef PICKLE_OK
#define PICKLE_OK              0
#define PICKLE_ERR_FORMAT     -1
#define PICKLE_ERR_VERSION    -2
#define PICKLE_ERR_MEMORY     -3
#define PICKLE_ERR_TYPE       -4
#define PICKLE_ERR_IO         -5
#define PICKLE_ERR_ARG        -6
#define PICKLE_ERR_RANGE      -7
#define PICKLE_ERR_ARCH       -8
#endif
/* New: a CUDA runtime error, a device-side bounded wait that gave up, or a
 * failed collective. The handle stays usable unless the CUDA context is
 * lost (pickle_cuda_last_error tells which). */
#define PICKLE_ERR_DEVICE     -9

#define PICKLE_CUDA_ABI_VERSION 1

#if defined(__GNUC__)
#define PICKLE_CUDA_API __attribute__((visibility("default")))
#else
#define PICKLE_CUDA_API
#endif

typedef struct pickle_cuda pickle_cuda_t;

/* Model dimensions the attention block needs. The fields mirror
 * pickle_fast_state_t (src/pickle_fast.h:55-123): n_layers, n_heads,
 * n_kv_heads, head_dim, max_seq, half, rope_inv_freq. */
typedef struct {
    int          n_layers;      /* state->n_layers */
    int          n_heads;       /* H: query heads */
    int          n_kv_heads;    /* HK: KV heads; H % HK == 0 */
    int          head_dim;      /* D: multiple of 4 (16-byte rows) */
    int          max_seq;       /* positions per sequence slot */
    int          half;          /* RoPE pairs per head: state->half = min(D/2, 64) */
    const float* rope_inv_freq; /* host [half]: state->rope_inv_freq (src/pickle_fast.c:1638-1640);
                                   NULL -> computed as 1/powf(theta, 2i/D) */
    float        rope_theta;    /* used only when rope_inv_freq == NULL */
    int          n_seqs;        /* sequence slots in the device cache (1 for pickle_fast_forward) */
    int          rope_len;      /* RoPE table rows (absolute positions); 0 = max_seq. A
                                   sequence-chunk shard holds max_seq cache rows but
                                   rotates at absolute positions up to rope_len - 1. */
} pickle_cuda_params_t;

/* Create a handle on CUDA device `device`: allocates the device KV cache
 * (zeroed, as calloc at src/pickle_fast.c:1793-1811), builds the RoPE
 * sin/cos table for positions [0, max_seq) on the host exactly as
 * pickle_fast_state_extend_rope does (src/pickle_fast.c:1772-1788) and
 * uploads it. Replaces pickle_fast_kv_alloc for the attention path.
 * Returns PICKLE_ERR_ARG on bad dimensions, PICKLE_ERR_MEMORY or
 * PICKLE_ERR_DEVICE on allocation / CUDA failure. */
PICKLE_CUDA_API int  pickle_cuda_init(const pickle_cuda_params_t* params, int device, pickle_cuda_t** out);
PICKLE_CUDA_API void pickle_cuda_free(pickle_cuda_t* h);

/* One decode step of one layer for sequence slot 0, host buffers.
 * Replaces src/pickle_fast.c:1910-2094 for one token:
 *   q [H*D] and k [HK*D] are rotated by RoPE at `pos` (not written back),
 *   rotated k and v [HK*D] are appended to the device cache at `pos`,
 *   ao [H*D] = softmax(q_h . K[0..pos] / sqrtf(D)) V[0..pos] per head h,
 *   with kv_head = h * HK / H (src/pickle_fast.c:1963).
 * Returns PICKLE_ERR_RANGE when pos >= max_seq (src/pickle_fast.c:1885). */
PICKLE_CUDA_API int  pickle_cuda_attn_decode(pickle_cuda_t* h, int layer, size_t pos,
                             const float* q, const float* k, const float* v,
                             float* ao);

/* Causal prefill of T tokens at positions [pos0, pos0+T) of sequence slot 0,
 * host buffers: q [T][H*D], k/v [T][HK*D], ao [T][H*D]. Same result as T
 * calls of pickle_cuda_attn_decode (the reference runs prefill token by
 * token, src/pickle_fast.c:1881), computed as one batched causal kernel.
 * `precision` selects PICKLE_CUDA_PREFILL_F32 (CUDA-core, FP32 parity) or
 * PICKLE_CUDA_PREFILL_BF16 (tensor cores, BF16 operands, F32 accumulate). */
#define PICKLE_CUDA_PREFILL_F32  0
#define PICKLE_CUDA_PREFILL_BF16 1
PICKLE_CUDA_API int  pickle_cuda_attn_prefill(pickle_cuda_t* h, int layer, size_t pos0, size_t T,
                              const float* q, const float* k, const float* v,
                              float* ao, int precision);

/* Batched decode over device buffers on `stream` (a cudaStream_t, NULL =
 * legacy default stream). All n_seqs sequences decode at the same `pos`:
 *   q  [n_seqs][H][D], k/v [n_seqs][HK][D] (pre-RoPE), ao [n_seqs][H][D].
 * Asynchronous: returns after the launch; errors of the launch itself are
 * returned, device-side wait timeouts are reported by pickle_cuda_sync. */
PICKLE_CUDA_API int  pickle_cuda_decode_batch_dev(pickle_cuda_t* h, int layer, int n_seqs, size_t pos,
                                  const float* q, const float* k, const float* v,
                                  float* ao, void* stream);

/* Batched causal prefill over device buffers on `stream`, positions
 * [pos0, pos0+T) of each of n_seqs sequences:
 *   q [n_seqs][T][H][D], k/v [n_seqs][T][HK][D] (pre-RoPE, F32),
 *   ao [n_seqs][T][H][D] (F32). The rotated k and v are written to the
 *   device cache for later decode. */
PICKLE_CUDA_API int  pickle_cuda_prefill_dev(pickle_cuda_t* h, int layer, int n_seqs, size_t pos0, size_t T,
                             const float* q, const float* k, const float* v,
                             float* ao, int precision, void* stream);

/* Causal attention only, on already rotated BF16 operands in head-major
 * layout: q [n_seqs][H][T][D], k/v [n_seqs][HK][T][D] (BF16), output
 * ao [n_seqs][T][H][D] F32; query t attends keys [0, t]. The tensor-core
 * kernel that pickle_cuda_prefill_dev runs after its RoPE/cast/cache-write
 * producer, exposed for callers whose activations are already BF16.
 * head_dim must be 128. err_flag (optional device int) records a device
 * wait that gave up. */
PICKLE_CUDA_API int pickle_cuda_prefill_attn_bf16_dev(int n_seqs, int T, int n_heads, int n_kv_heads, int head_dim,
                                                      const void* q_bf16, const void* k_bf16, const void* v_bf16,
                                                      float* ao, int* err_flag, void* stream);

/* Partial decode for sequence-chunk sharding: the n_seqs queries at
 * absolute position `pos` (RoPE row) attend over the `n_local` cache rows
 * [0, n_local) this handle holds for each sequence; when append != 0 the
 * new (rotated) k/v are first stored at local row n_local and attended as
 * well. Writes, per (seq, head), the unnormalised triple
 *   m = max score, l = sum exp(s - m), acc[D] = sum exp(s - m) v
 * into m_out/l_out [n_seqs][H] and acc_out [n_seqs][H][D]. Merge the
 * triples of all shards with pickle_cuda_lse_merge_dev. */
PICKLE_CUDA_API int  pickle_cuda_decode_partial_dev(pickle_cuda_t* h, int layer, int n_seqs, size_t pos,
                                    size_t n_local, int append,
                                    const float* q, const float* k, const float* v,
                                    float* m_out, float* l_out, float* acc_out, void* stream);

/* Ragged decode for continuous batching (no counterpart in the reference,
 * which decodes one sequence at a time): entry i of the batch (i < n) is
 * the sequence in cache slot slot_dev[i] (slot_dev NULL: slot i) at its
 * own position pos_dev[i] - it attends rows [0, pos_dev[i]) of that slot,
 * rotates q and k with table row pos_dev[i] and appends k, v there, exactly
 * as pickle_cuda_decode_batch_dev does for one position. pos_dev and
 * slot_dev are device int arrays; max_pos (host) bounds every pos_dev[i]
 * and must be < max_seq and < the RoPE table length (PICKLE_ERR_RANGE). An
 * entry whose position exceeds max_pos or whose slot is outside
 * [0, n_seqs) is skipped and recorded as a device error, reported by
 * pickle_cuda_sync. Slots within one call must be distinct.
 * q [n][H][D], k/v [n][HK][D], ao [n][H][D]. */
PICKLE_CUDA_API int  pickle_cuda_decode_ragged_dev(pickle_cuda_t* h, int layer, int n, const int* pos_dev,
                                                   const int* slot_dev, size_t max_pos, const float* q,
                                                   const float* k, const float* v, float* ao, void* stream);

/* pickle_cuda_prefill_dev for the one sequence in cache slot `slot` (no
 * counterpart in the reference): the prompt of a request admitted into a
 * free slot of a continuously batched decode. q [T][H][D], k/v [T][HK][D],
 * ao [T][H][D]. */
PICKLE_CUDA_API int  pickle_cuda_prefill_slot_dev(pickle_cuda_t* h, int layer, int slot, size_t pos0, size_t T,
                                                  const float* q, const float* k, const float* v, float* ao,
                                                  int precision, void* stream);

/* Log-sum-exp merge of n_parts partial triples laid out
 * [n_parts][n_rows] (m, l) and [n_parts][n_rows][D] (acc):
 *   M = max_i m_i,  o = sum_i e^(m_i - M) acc_i / sum_i e^(m_i - M) l_i. */
PICKLE_CUDA_API int  pickle_cuda_lse_merge_dev(int n_parts, int n_rows, int head_dim,
                               const float* m_in, const float* l_in, const float* acc_in,
                               float* out, void* stream);

/* Decode without any allocation, for callers that cannot let a library
 * call cudaMalloc (their device memory comes from their own arena). No
 * counterpart in the reference. Same computation as
 * pickle_cuda_decode_batch_dev on caller-owned device buffers: q [n_seqs][H][D],
 * k/v [n_seqs][HK][D] (pre-RoPE), the head-major cache
 * k_cache/v_cache [n_seqs][HK][max_seq][D] (row pos is written), RoPE tables
 * rope_sin/rope_cos [>= pos+1][half] and ao [n_seqs][H][D]; err_flag is an
 * optional device int that records a bounded wait giving up. Its split-KV
 * scratch is a fixed 4 MiB device array inside this library, shared by all
 * calls: calls that overlap on the GPU race, so serialise them on one
 * stream. n_seqs * n_kv_heads above 4096 is rejected (PICKLE_ERR_RANGE).
 * Uses the current device; its first call there does a one-time set-up
 * (looks up the array's address) and should come before any stream capture. */
PICKLE_CUDA_API int pickle_cuda_decode_noalloc(int n_seqs, int n_heads, int n_kv_heads, int head_dim,
                                               int half, int max_seq, size_t pos,
                                               const float* rope_sin, const float* rope_cos,
                                               const float* q, const float* k, const float* v,
                                               float* k_cache, float* v_cache, float* ao,
                                               int* err_flag, void* stream);

/* The same merge over parts packed back to back, as one all-gather of
 * per-rank buffers leaves them: part i starts at parts + i * part_stride
 * (floats, >= n_rows * (head_dim + 2)) and holds acc [n_rows][head_dim],
 * then m [n_rows], then l [n_rows]. A rank fills its part by passing
 * acc_out = part, m_out = part + n_rows * head_dim, l_out = m_out + n_rows
 * to pickle_cuda_decode_partial_dev. */
PICKLE_CUDA_API int pickle_cuda_lse_merge_packed_dev(int n_parts, int n_rows, int head_dim, const float* parts,
                                                     size_t part_stride, float* out, void* stream);

/* Copy host K/V rows in pickle's own layout [n_pos][HK][D] (already
 * rotated, as the host cache holds them) into the device cache at
 * positions [pos0, pos0+n_pos) of (layer, seq). Lets a caller import a
 * host pickle_fast_kv_t. */
PICKLE_CUDA_API int  pickle_cuda_kv_write(pickle_cuda_t* h, int layer, int seq, size_t pos0, size_t n_pos,
                          const float* k_host, const float* v_host);

/* Device addresses of layer `layer`'s cache, for callers that fill or
 * inspect it with their own kernels; *seq_stride, *head_stride are in
 * floats (row stride is head_dim). */
PICKLE_CUDA_API int  pickle_cuda_kv_layout(pickle_cuda_t* h, int layer, float** k_dev, float** v_dev,
                           size_t* seq_stride, size_t* head_stride);

/* Wait for all work on `stream` and report device-side errors (a bounded
 * wait that gave up) recorded since the last call. */
PICKLE_CUDA_API int  pickle_cuda_sync(pickle_cuda_t* h, void* stream);

/* Number of KV splits the decode launch uses for (n_seqs, pos) on this
 * handle, and how many kernels it launches (the split kernel, plus the merge
 * kernel when there is more than one split). */
PICKLE_CUDA_API int  pickle_cuda_decode_plan(pickle_cuda_t* h, int n_seqs, size_t pos, int* n_splits,
                             int* n_launches);

/* Last CUDA error string seen by this handle (never NULL). */
PICKLE_CUDA_API const char* pickle_cuda_last_error(pickle_cuda_t* h);

PICKLE_CUDA_API int  pickle_cuda_abi_version(void);

/* ---- Projections either side of the attention block ----
 * y[v][o] = sum_i W[o][i] * x[v][i] for v < n_vec (1..8 vectors sharing one
 * pass over W), with W [out_n][in_n] in its raw on-disk layout of GGML type
 * `type`: 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 12 Q4_K, 14 Q6_K (the values of
 * src/pickle.h:85-97). Replaces pickle_fast_matmul_dispatch
 * (src/pickle_fast.c:1423-1474) for those types, with the same per-weight
 * dequantization and a float activation (the reference's float paths);
 * other types return PICKLE_ERR_TYPE like the dispatch. in_n must be a
 * multiple of the type's block (4, 32 or 256 elements); W, x and y
 * 16-byte aligned device buffers; x [n_vec][in_n], y [n_vec][out_n]. */
#define PICKLE_CUDA_MATVEC_MAX_VEC 8
PICKLE_CUDA_API int  pickle_cuda_matvec_dev(int type, const void* W, int out_n, int in_n, int n_vec,
                                            const float* x, float* y, void* stream);
/* Bytes of one W row of `type` for in_n elements (0: unsupported or not a
 * whole number of blocks). */
PICKLE_CUDA_API size_t pickle_cuda_matvec_row_bytes(int type, int in_n);
/* The device error word of the tensor-core matvec on `device` (a bounded
 * wait that gave up: PCU_DEVERR codes 1-3, 0 = none), read and cleared.
 * Synchronous. No reference counterpart (the reference has no device). */
PICKLE_CUDA_API int  pickle_cuda_matvec_take_error(int device, int* code);

/* ---- The same projections for many activation rows (batched prefill) ----
 * y[t][o] = sum_i W[o][i] * x[t][i] for t < n_tok: the reference's per-token
 * pickle_fast_matmul_dispatch (src/pickle_fast.c:1423-1474, called once per
 * token from the layer loop, :1903-1907, :2112, :2120-2133) for a whole
 * prompt. With more than PICKLE_CUDA_MATVEC_MAX_VEC rows, F16, Q8_0, Q4_0,
 * Q4_K and Q6_K weights whose rows are 16-byte multiples, with in_n a
 * multiple of 256, go through a tensor-core GEMM that needs a caller-owned
 * device workspace of pickle_cuda_matmul_workspace(out_n, in_n, n_tok) bytes
 * (256-byte aligned); every other case (or workspace == NULL) runs the
 * matvec over the rows in passes of eight. Same types, alignment and status
 * codes as the matvec. */
PICKLE_CUDA_API size_t pickle_cuda_matmul_workspace(int out_n, int in_n, int n_tok);
PICKLE_CUDA_API int  pickle_cuda_matmul_dev(int type, const void* W, int out_n, int in_n, int n_tok,
                                            const float* x, float* y, void* workspace, size_t ws_bytes,
                                            void* stream);

/* ---- The whole forward pass on the device ----
 * Replaces pickle_fast_state_init + pickle_fast_forward
 * (src/pickle_fast.c:1497-1662, 1822-2184) and the greedy decode loop of
 * pickle_chat_loop (src/pickle_host.c:473-521) for Llama-family GGUF models.
 * A model is loaded from the same tensors pickle_fast_state_init finds by
 * name (:1530-1633); each is its raw GGML bytes, [out][in] as on disk. */
typedef struct pickle_cuda_model pickle_cuda_model_t;

typedef struct {
    int         type;    /* GGML type: 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 12 Q4_K, 14 Q6_K */
    const void* data;    /* host bytes, or device bytes when weights_on_device; NULL = absent */
    size_t      nbytes;  /* must equal rows * pickle_cuda_matvec_row_bytes(type, cols) */
} pickle_cuda_tensor_t;

/* Per-layer tensors, in this order ("blk.<L>.<name>.weight"):
 * attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate,
 * ffn_up, ffn_down. Norm weights are F32. */
#define PICKLE_CUDA_LAYER_TENSORS 9

typedef struct {
    int   n_layers, hidden_dim, intermediate_dim;   /* state->n_layers, hidden_dim, intermediate_dim */
    int   n_heads, n_kv_heads, head_dim;            /* H, HK, D (D a multiple of 4) */
    int   vocab_size, max_seq;                      /* VS, cache positions (arch->max_seq_len) */
    float rms_eps, rope_theta;                      /* state->rms_eps; theta when rope_inv_freq is NULL */
    const float* rope_inv_freq;                     /* host [min(D/2, 64)] or NULL, as pickle_cuda_params_t */
    int   max_tokens;         /* prompt tokens per device pass (activation buffers and GEMM workspace
                                 are sized for it); longer prompts run in chunks */
    int   prefill_precision;  /* PICKLE_CUDA_PREFILL_F32 (parity) or PICKLE_CUDA_PREFILL_BF16 */
    int   weights_on_device;  /* 0: data are host pointers, copied into one device allocation at load;
                                 1: data are 16-byte aligned device pointers used in place (the caller
                                 keeps them alive until pickle_cuda_model_free) */
    pickle_cuda_tensor_t token_embd;   /* "token_embd.weight" [vocab][hidden]: F32 or F16 rows are looked
                                          up as they are; Q4_0, Q8_0, Q4_K, Q6_K are dequantized to an
                                          F32 table at load, as pickle_fast_state_init does (:1551-1584) */
    pickle_cuda_tensor_t output_norm;  /* "output_norm.weight", F32 [hidden]; NULL = no final norm */
    pickle_cuda_tensor_t output;       /* "output.weight" [vocab][hidden]; NULL = token_embd (tied) */
    const pickle_cuda_tensor_t* layers; /* [n_layers][PICKLE_CUDA_LAYER_TENSORS] */
    int   n_seqs;             /* sequence slots in the device KV cache (0 or 1: one, as the reference) */
} pickle_cuda_model_params_t;

/* Uploads the weights and allocates the device KV cache (one sequence),
 * the activations and the GEMM workspace. PICKLE_ERR_ARCH: a required
 * tensor is missing; PICKLE_ERR_TYPE: a type the device path does not run;
 * PICKLE_ERR_ARG: a size that does not match the dimensions. */
PICKLE_CUDA_API int  pickle_cuda_model_load(const pickle_cuda_model_params_t* params, int device,
                                            pickle_cuda_model_t** out);
PICKLE_CUDA_API void pickle_cuda_model_free(pickle_cuda_model_t* m);
/* The attention handle inside the model (its KV cache, decode plan). */
PICKLE_CUDA_API pickle_cuda_t* pickle_cuda_model_attn(pickle_cuda_model_t* m);
PICKLE_CUDA_API const char* pickle_cuda_model_last_error(pickle_cuda_model_t* m);

/* pickle_fast_forward with host buffers: n_tokens tokens at positions
 * *kv_pos .. *kv_pos + n_tokens - 1; out_logits [vocab] gets the last
 * token's logits; *kv_pos advances by n_tokens. Synchronous.
 * PICKLE_ERR_RANGE for a token outside [0, vocab) or a position >= max_seq
 * (nothing is computed and *kv_pos is kept, as the reference keeps it). */
PICKLE_CUDA_API int  pickle_cuda_forward(pickle_cuda_model_t* m, const int32_t* tokens, size_t n_tokens,
                                         float* out_logits, size_t* kv_pos);
/* pickle_cuda_forward for the sequence in cache slot `slot` (0 <= slot <
 * n_seqs; no counterpart in the reference, which serves one conversation
 * per KV cache): the prompt of a request admitted into a free slot, or one
 * of its tokens. PICKLE_ERR_RANGE for a slot outside the model's. */
PICKLE_CUDA_API int  pickle_cuda_forward_slot(pickle_cuda_model_t* m, int slot, const int32_t* tokens,
                                              size_t n_tokens, float* out_logits, size_t* kv_pos);
/* One decode step of n sequences together (continuous batching; no
 * counterpart in the reference): sequence i feeds token tokens_dev[i] at
 * position pos_dev[i] of cache slot slot_dev[i] (device int arrays; slots
 * distinct, positions <= max_pos < max_seq). All n rows go through each
 * projection in one pass over the weights. logits_dev [n][vocab] gets every
 * row's logits (vocab a multiple of 4 when n > 1), next_dev [n] (optional)
 * their pickle_fast_argmax ids. Asynchronous on `stream`; a position or slot
 * out of range is a device error reported by pickle_cuda_model_sync. */
PICKLE_CUDA_API int  pickle_cuda_forward_batch_dev(pickle_cuda_model_t* m, int n, const int32_t* tokens_dev,
                                                   const int* pos_dev, const int* slot_dev, size_t max_pos,
                                                   float* logits_dev, int32_t* next_dev, void* stream);
/* The same on device buffers, asynchronous on `stream`: tokens_dev [n_tokens]
 * at positions pos0.., logits_dev [vocab] (last token), and, when next_dev is
 * not NULL, its pickle_fast_argmax id in *next_dev. Device-side errors (a token
 * id out of range, a bounded wait that gave up) are reported by
 * pickle_cuda_model_sync. */
PICKLE_CUDA_API int  pickle_cuda_forward_dev(pickle_cuda_model_t* m, const int32_t* tokens_dev, size_t n_tokens,
                                             size_t pos0, float* logits_dev, int32_t* next_dev, void* stream);
PICKLE_CUDA_API int  pickle_cuda_model_sync(pickle_cuda_model_t* m, void* stream);
/* pickle_fast_argmax (src/pickle_fast.c:2186-2194) on the device: the first
 * index holding the largest value, as a scan that keeps the first strictly
 * larger one finds it (so 0 when logits[0] is NaN, other NaNs never win).
 * logits [n] and out (one int32) are device buffers; asynchronous. */
PICKLE_CUDA_API int  pickle_cuda_argmax_dev(const float* logits, int n, int32_t* out, void* stream);
/* pickle_fast_sample_temp (src/pickle_fast.c:2204-2276) on the device, one
 * CTA: temp <= 0 is the argmax; otherwise softmax(logits / temp) (logits is
 * overwritten with the unnormalized exponentials, as the reference does),
 * one xorshift32 draw from seed (0 -> 0x12345678), and top-p (nucleus)
 * sampling when 0 < top_p < 1, else plain temperature sampling. The sums
 * are fixed-order trees, not the reference's one running float sum: a draw
 * within float rounding of a probability boundary may pick the neighbouring
 * id. Ties in probability go to the lower index. Asynchronous. */
PICKLE_CUDA_API int  pickle_cuda_sample_dev(float* logits, int n, float temp, float top_p, uint32_t seed,
                                            int32_t* out, void* stream);
/* Greedy generation as pickle_chat_loop runs it with temp <= 0: forward the
 * prompt, then n_gen times take the argmax id, stop after eos_id (>= 0;
 * -1 = none) or when the cache is full, else forward that id. The ids stay
 * on the device between steps. out_ids [n_gen] gets *n_out ids, last_logits
 * [vocab] (optional) the logits the last id was taken from, or those after
 * its forward when it was forwarded, and *kv_pos the next free position. */
PICKLE_CUDA_API int  pickle_cuda_generate(pickle_cuda_model_t* m, const int32_t* prompt, size_t n_prompt,
                                          int n_gen, int eos_id, int32_t* out_ids, int* n_out,
                                          float* last_logits, size_t* kv_pos);
/* The same loop with pickle_chat_loop's sampler: id i is
 * pickle_fast_sample_temp(logits, vocab, temp, top_p, seed + i) (greedy when
 * temp <= 0), run on the device (pickle_cuda_sample_dev). The sampler
 * leaves the logits it sampled from as expf(logits / temp - max), as the
 * reference's does. */
PICKLE_CUDA_API int  pickle_cuda_generate_sampled(pickle_cuda_model_t* m, const int32_t* prompt, size_t n_prompt,
                                                  int n_gen, int eos_id, float temp, float top_p, uint32_t seed,
                                                  int32_t* out_ids, int* n_out, float* last_logits, size_t* kv_pos);

/* ---- Peer exchange of the sharded decodes (one process per GPU) ----
 * No counterpart in the reference, which runs on one host: this replaces an
 * NCCL all-gather for the small per-step payloads of the KV-head and
 * sequence-chunk shards. Each rank creates an exchange with the same
 * buf_bytes, shares pickle_cuda_xchg_handle's bytes with the other ranks
 * (any host-side all-gather) and opens theirs. pickle_cuda_xchg_put_dev then
 * copies `rows` rows of row_bytes (16-byte multiples) from this rank's src
 * into every rank's receive buffer (pickle_cuda_xchg_buffer) at
 * dst_offset + r * dst_stride, and completes on the GPU once every rank's
 * rows of this call have arrived in this rank's buffer. A call first waits
 * until each destination rank has started the same call, so a rank never
 * overwrites rows another rank has not consumed (consume them on the stream
 * that makes the next call). All ranks make the same sequence of calls; a
 * rank that stops turns into an error (pickle_cuda_xchg_sync) on the others
 * after a bounded 1 s wait. Plain peer stores through CUDA IPC mappings, no
 * multicast; the call counters live on the device. */
#define PICKLE_CUDA_XCHG_MAX_RANKS 8
#define PICKLE_CUDA_IPC_HANDLE_BYTES 64
typedef struct pickle_cuda_xchg pickle_cuda_xchg_t;
PICKLE_CUDA_API int  pickle_cuda_xchg_create(int rank, int world, size_t buf_bytes, int device,
                                             pickle_cuda_xchg_t** out);
PICKLE_CUDA_API int  pickle_cuda_xchg_handle(pickle_cuda_xchg_t* x, void* handle_out);
PICKLE_CUDA_API int  pickle_cuda_xchg_open(pickle_cuda_xchg_t* x, int peer, const void* handle);
PICKLE_CUDA_API int  pickle_cuda_xchg_buffer(pickle_cuda_xchg_t* x, void** dev_ptr);
PICKLE_CUDA_API int  pickle_cuda_xchg_put_dev(pickle_cuda_xchg_t* x, const void* src, size_t rows,
                                              size_t row_bytes, size_t src_stride, size_t dst_offset,
                                              size_t dst_stride, void* stream);
/* Reports a bounded wait of this rank's exchanging kernels that gave up
 * (PICKLE_ERR_DEVICE). The exchange is then broken - the ranks' call
 * counters no longer agree - and every later call on it returns
 * PICKLE_ERR_DEVICE: free it and create a new one on every rank. */
PICKLE_CUDA_API int  pickle_cuda_xchg_sync(pickle_cuda_xchg_t* x, void* stream);
PICKLE_CUDA_API const char* pickle_cuda_xchg_last_error(pickle_cuda_xchg_t* x);
PICKLE_CUDA_API void pickle_cuda_xchg_free(pickle_cuda_xchg_t* x);

/* Ranks driven by one process (one exchange per rank, on its own GPU, or
 * several on one GPU for tests) use each other's regions directly instead
 * of through IPC handles: rank `peer`'s exchange `other` becomes x's peer.
 * Devices must be able to reach each other (peer access is enabled). */
PICKLE_CUDA_API int  pickle_cuda_xchg_attach(pickle_cuda_xchg_t* x, int peer, pickle_cuda_xchg_t* other);

/* Bound of every flag wait of this exchange's kernels, in nanoseconds
 * (default 1 s). */
PICKLE_CUDA_API int  pickle_cuda_xchg_set_wait(pickle_cuda_xchg_t* x, unsigned long long wait_ns);

/* ---- Sharded decodes with the exchange fused into the launch ----
 * No counterpart in the reference (one host, OpenMP over heads,
 * src/pickle_fast.c:1960). Each is two launches on `stream`: the split-KV
 * decode of this rank's share, then one kernel that merges its splits,
 * stores the result straight into every rank's exchange buffer with plain
 * peer stores (no multicast) as epoch-tagged words, and assembles this
 * rank's output from what all ranks stored - no fence, flag or extra
 * launch. All ranks make the same calls with the same n_seqs; q/k/v are
 * this rank's inputs as for pickle_cuda_decode_batch_dev /
 * pickle_cuda_decode_partial_dev. The exchange buffer must hold
 * pickle_cuda_decode_xchg_bytes(...) bytes (calls alternate between its
 * two halves). Decode errors are reported by pickle_cuda_sync(h), exchange
 * waits that gave up by pickle_cuda_xchg_sync(x). n_seqs * n_heads (of
 * this handle) <= 4096.
 *
 * KV-head shard: this handle holds this rank's KV heads and their n_heads
 * query heads (kv_head = h * HK / H keeps them together,
 * src/pickle_fast.c:1963); rank r's heads are [r * n_heads, (r+1) * n_heads)
 * of the model. out [n_seqs][world * n_heads][head_dim] (this rank's device
 * memory) receives every rank's head outputs. */
#define PICKLE_CUDA_SHARD_HEADS 0
#define PICKLE_CUDA_SHARD_SEQ   1
PICKLE_CUDA_API int  pickle_cuda_decode_gather_dev(pickle_cuda_t* h, pickle_cuda_xchg_t* x, int layer, int n_seqs,
                                                   size_t pos, const float* q, const float* k, const float* v,
                                                   float* out, void* stream);

/* Sequence-chunk shard: this handle holds this rank's n_local cache rows
 * of every sequence (append != 0 on the rank that also stores the new
 * token at local row n_local); queries rotate at absolute position pos.
 * The triples (max, sum, acc) of every rank are exchanged and merged by
 * log-sum-exp into out [n_seqs][n_heads][head_dim] (this rank's device
 * memory). */
PICKLE_CUDA_API int  pickle_cuda_decode_seqshard_dev(pickle_cuda_t* h, pickle_cuda_xchg_t* x, int layer,
                                                     int n_seqs, size_t pos, size_t n_local, int append,
                                                     const float* q, const float* k, const float* v, float* out,
                                                     void* stream);

/* Exchange buffer bytes the fused sharded decodes need:
 * sharding = PICKLE_CUDA_SHARD_HEADS (n_heads = this rank's query heads)
 * or PICKLE_CUDA_SHARD_SEQ (n_heads = all query heads). */
PICKLE_CUDA_API int  pickle_cuda_decode_xchg_bytes(int sharding, int world, int n_seqs, int n_heads, int head_dim,
                                                   size_t* bytes);

#ifdef __cplusplus
}
#endif
#endif /* PICKLE_CUDA_H */
