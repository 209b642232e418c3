/*
 * ref_attn_cpu.c - CPU restatement of pickle's per-layer attention block.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity oracle: tests, the
 * smoke check and bench.py's CPU-baseline leg call it to check or time
 * against. The product (lestramanika_b200/csrc) never links it.
 *
 * It restates, for one token of one layer, what
 * lee-muriithi-kingori/lestramanika src/pickle_fast.c does at
 *   :1634-1640  inv_freq[i] = 1 / powf(theta, (float)(2i) / (float)D)
 *   :1772-1788  sin/cos[pos*half + i] = sinf/cosf(inv_freq[i] * (float)pos)
 *   :1910-1936  NeoX RoPE on the pairs (x[i], x[i+half]) of every q and k head
 *   :1938-1944  append k, v to the pos-major cache [layer][pos][kv_head][D]
 *   :1958-2094  per query head: scores over [0, pos] scaled by 1/sqrtf(D),
 *               softmax (max, expf, sum, sum==0 -> 1), weighted sum of V
 * with the same floating-point operation order (4-accumulator AVX-512 dot
 * for D % 16 == 0, `omp simd` reductions otherwise), so that with the same
 * compiler flags its outputs are bit-identical to the reference's. That
 * claim is checked by the test suite against the reference's own block,
 * compiled from its sources into oracle/_ref.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#if defined(__AVX512F__)
#include <immintrin.h>
#endif

typedef struct oracle_attn {
    int    n_layers, n_heads, n_kv_heads, head_dim, max_seq, half;
    float* inv_freq;     /* [half] */
    float* rope_sin;     /* [max_seq][half] */
    float* rope_cos;     /* [max_seq][half] */
    float* k_cache;      /* [n_layers][max_seq][n_kv_heads][head_dim] */
    float* v_cache;
    size_t layer_stride; /* max_seq * n_kv_heads * head_dim */
} oracle_attn_t;

#define ORACLE_OK         0
#define ORACLE_ERR_MEMORY -3
#define ORACLE_ERR_ARG    -6
#define ORACLE_ERR_RANGE  -7

/* RoPE tables, src/pickle_fast.c:1634-1640 and :1772-1788. `half` follows
 * src/pickle_fast.c:1515-1516 (head_dim / 2, capped at 64). */
int oracle_rope_tables(float theta, int head_dim, int half, int n_pos,
                       float* inv_freq, float* sin_tab, float* cos_tab) {
    if (head_dim <= 0 || half < 0 || n_pos < 0) return ORACLE_ERR_ARG;
    for (int i = 0; i < half; i++)
        inv_freq[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
    for (int p = 0; p < n_pos; p++) {
        for (int i = 0; i < half; i++) {
            float angle = inv_freq[i] * (float)p;
            sin_tab[(size_t)p * half + i] = sinf(angle);
            cos_tab[(size_t)p * half + i] = cosf(angle);
        }
    }
    return ORACLE_OK;
}

int oracle_attn_create(int n_layers, int n_heads, int n_kv_heads, int head_dim,
                       int max_seq, float theta, oracle_attn_t** out) {
    if (!out || n_layers <= 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 ||
        max_seq <= 0 || n_heads % n_kv_heads)
        return ORACLE_ERR_ARG;
    oracle_attn_t* o = (oracle_attn_t*)calloc(1, sizeof(*o));
    if (!o) return ORACLE_ERR_MEMORY;
    o->n_layers = n_layers; o->n_heads = n_heads; o->n_kv_heads = n_kv_heads;
    o->head_dim = head_dim; o->max_seq = max_seq;
    o->half = head_dim / 2 > 64 ? 64 : head_dim / 2;
    o->layer_stride = (size_t)max_seq * n_kv_heads * head_dim;
    size_t tab = (size_t)max_seq * (o->half ? o->half : 1);
    o->inv_freq = (float*)calloc(o->half ? o->half : 1, sizeof(float));
    o->rope_sin = (float*)calloc(tab, sizeof(float));
    o->rope_cos = (float*)calloc(tab, sizeof(float));
    o->k_cache  = (float*)calloc((size_t)n_layers * o->layer_stride, sizeof(float));
    o->v_cache  = (float*)calloc((size_t)n_layers * o->layer_stride, sizeof(float));
    if (!o->inv_freq || !o->rope_sin || !o->rope_cos || !o->k_cache || !o->v_cache) {
        free(o->inv_freq); free(o->rope_sin); free(o->rope_cos);
        free(o->k_cache); free(o->v_cache); free(o);
        return ORACLE_ERR_MEMORY;
    }
    oracle_rope_tables(theta, head_dim, o->half, max_seq, o->inv_freq, o->rope_sin, o->rope_cos);
    *out = o;
    return ORACLE_OK;
}

void oracle_attn_destroy(oracle_attn_t* o) {
    if (!o) return;
    free(o->inv_freq); free(o->rope_sin); free(o->rope_cos);
    free(o->k_cache); free(o->v_cache); free(o);
}

float* oracle_attn_k_cache(oracle_attn_t* o) { return o->k_cache; }
float* oracle_attn_v_cache(oracle_attn_t* o) { return o->v_cache; }
float* oracle_attn_sin(oracle_attn_t* o) { return o->rope_sin; }
float* oracle_attn_cos(oracle_attn_t* o) { return o->rope_cos; }
float* oracle_attn_inv_freq(oracle_attn_t* o) { return o->inv_freq; }

/* Rotate n_heads heads of x [n_heads][D] in place with one table row
 * (src/pickle_fast.c:1913-1936). */
static void rope_rotate(float* x, int n_heads, int D, int half,
                        const float* sin_row, const float* cos_row) {
    for (int h = 0; h < n_heads; h++) {
        float* xh = x + (size_t)h * D;
        for (int i = 0; i < half; i++) {
            float lo = xh[i];
            float hi = xh[i + half];
            float c = cos_row[i], s = sin_row[i];
            xh[i]        = c * lo - s * hi;
            xh[i + half] = s * lo + c * hi;
        }
    }
}

/* q . k for one cached row, src/pickle_fast.c:1980-2032. */
static inline float row_dot(const float* a, const float* b, int D) {
#if defined(__AVX512F__)
    if ((D & 15) == 0) {
        __m512 s0 = _mm512_setzero_ps(), s1 = _mm512_setzero_ps();
        __m512 s2 = _mm512_setzero_ps(), s3 = _mm512_setzero_ps();
        int d = 0;
        for (; d + 64 <= D; d += 64) {
            __m512 a0 = _mm512_loadu_ps(a + d),      a1 = _mm512_loadu_ps(a + d + 16);
            __m512 a2 = _mm512_loadu_ps(a + d + 32), a3 = _mm512_loadu_ps(a + d + 48);
            __m512 b0 = _mm512_loadu_ps(b + d),      b1 = _mm512_loadu_ps(b + d + 16);
            __m512 b2 = _mm512_loadu_ps(b + d + 32), b3 = _mm512_loadu_ps(b + d + 48);
            s0 = _mm512_fmadd_ps(a0, b0, s0);
            s1 = _mm512_fmadd_ps(a1, b1, s1);
            s2 = _mm512_fmadd_ps(a2, b2, s2);
            s3 = _mm512_fmadd_ps(a3, b3, s3);
        }
        for (; d + 16 <= D; d += 16)
            s0 = _mm512_fmadd_ps(_mm512_loadu_ps(a + d), _mm512_loadu_ps(b + d), s0);
        __m512 t = _mm512_add_ps(_mm512_add_ps(s0, s1), _mm512_add_ps(s2, s3));
        float r = _mm512_reduce_add_ps(t);
        for (; d < D; d++) r += a[d] * b[d];
        return r;
    }
#endif
    float r = 0.0f;
    #pragma omp simd reduction(+:r)
    for (int d = 0; d < D; d++) r += a[d] * b[d];
    return r;
}

/* o += w * v for one cached row, src/pickle_fast.c:2046-2091. */
static inline void row_axpy(float* o, float w, const float* v, int D) {
#if defined(__AVX512F__)
    if ((D & 15) == 0) {
        __m512 wv = _mm512_set1_ps(w);
        int d = 0;
        for (; d + 64 <= D; d += 64) {
            __m512 o0 = _mm512_fmadd_ps(wv, _mm512_loadu_ps(v + d),      _mm512_loadu_ps(o + d));
            __m512 o1 = _mm512_fmadd_ps(wv, _mm512_loadu_ps(v + d + 16), _mm512_loadu_ps(o + d + 16));
            __m512 o2 = _mm512_fmadd_ps(wv, _mm512_loadu_ps(v + d + 32), _mm512_loadu_ps(o + d + 32));
            __m512 o3 = _mm512_fmadd_ps(wv, _mm512_loadu_ps(v + d + 48), _mm512_loadu_ps(o + d + 48));
            _mm512_storeu_ps(o + d, o0);      _mm512_storeu_ps(o + d + 16, o1);
            _mm512_storeu_ps(o + d + 32, o2); _mm512_storeu_ps(o + d + 48, o3);
        }
        for (; d + 16 <= D; d += 16)
            _mm512_storeu_ps(o + d, _mm512_fmadd_ps(wv, _mm512_loadu_ps(v + d), _mm512_loadu_ps(o + d)));
        for (; d < D; d++) o[d] += w * v[d];
        return;
    }
#endif
    #pragma omp simd
    for (int d = 0; d < D; d++) o[d] += w * v[d];
}

/* Attention of query head h over cache rows [0, n) of one layer with an
 * explicit row stride; `scores` has room for n floats. */
static void head_attend(const float* qh, const float* kbase, const float* vbase,
                        size_t row_stride, size_t n, int D, float scale,
                        float* scores, float* oh) {
    for (size_t p = 0; p < n; p++)
        scores[p] = row_dot(qh, kbase + p * row_stride, D) * scale;
    float mx = scores[0];
    for (size_t p = 1; p < n; p++)
        if (scores[p] > mx) mx = scores[p];
    float total = 0.0f;
    for (size_t p = 0; p < n; p++) {
        scores[p] = expf(scores[p] - mx);
        total += scores[p];
    }
    if (total == 0.0f) total = 1.0f;
    float inv = 1.0f / total;
    for (int d = 0; d < D; d++) oh[d] = 0.0f;
    for (size_t p = 0; p < n; p++)
        row_axpy(oh, scores[p] * inv, vbase + p * row_stride, D);
}

/* One decode step: RoPE on q (H heads) and k (HK heads) in place at `pos`,
 * append k, v at `pos` of `layer`, attention over [0, pos] into ao [H*D]. */
int oracle_attn_decode(oracle_attn_t* o, int layer, size_t pos,
                       float* q, float* k, const float* v, float* ao) {
    if (!o || layer < 0 || layer >= o->n_layers || !q || !k || !v || !ao) return ORACLE_ERR_ARG;
    if (pos >= (size_t)o->max_seq) return ORACLE_ERR_RANGE;
    const int H = o->n_heads, HK = o->n_kv_heads, D = o->head_dim, half = o->half;
    if (half > 0) {
        const float* sr = o->rope_sin + pos * half;
        const float* cr = o->rope_cos + pos * half;
        rope_rotate(q, H, D, half, sr, cr);
        rope_rotate(k, HK, D, half, sr, cr);
    }
    float* kl = o->k_cache + (size_t)layer * o->layer_stride;
    float* vl = o->v_cache + (size_t)layer * o->layer_stride;
    memcpy(kl + pos * HK * D, k, (size_t)HK * D * sizeof(float));
    memcpy(vl + pos * HK * D, v, (size_t)HK * D * sizeof(float));

    const size_t n = pos + 1;
    const float scale = 1.0f / sqrtf((float)D);
    int err = 0;
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++) {
        float* scores = (float*)malloc(n * sizeof(float));
        if (!scores) { err = 1; continue; }
        int kvh = h * HK / H;
        head_attend(q + (size_t)h * D, kl + (size_t)kvh * D, vl + (size_t)kvh * D,
                    (size_t)HK * D, n, D, scale, scores, ao + (size_t)h * D);
        free(scores);
    }
    return err ? ORACLE_ERR_MEMORY : ORACLE_OK;
}

/* Batched variant used by the tests and the CPU baseline: n_seqs
 * independent sequences with their own pos-major caches
 * kc/vc [n_seqs][max_seq][HK][D] (the reference has no batch dimension,
 * so this is n_seqs sequential reference steps). q/k/v/ao are
 * [n_seqs][heads][D]; q and k are rotated in place. */
int oracle_attn_decode_batch(int n_seqs, int H, int HK, int D, int max_seq, size_t pos,
                             const float* sin_row, const float* cos_row,
                             float* kc, float* vc, float* q, float* k, const float* v,
                             float* ao) {
    if (pos >= (size_t)max_seq || H % HK) return ORACLE_ERR_ARG;
    const int half = D / 2 > 64 ? 64 : D / 2;
    const size_t n = pos + 1;
    const float scale = 1.0f / sqrtf((float)D);
    const size_t seq_stride = (size_t)max_seq * HK * D;
    int err = 0;
    for (int b = 0; b < n_seqs; b++) {
        float* qb = q + (size_t)b * H * D;
        float* kb = k + (size_t)b * HK * D;
        rope_rotate(qb, H, D, half, sin_row, cos_row);
        rope_rotate(kb, HK, D, half, sin_row, cos_row);
        float* kl = kc + (size_t)b * seq_stride;
        float* vl = vc + (size_t)b * seq_stride;
        memcpy(kl + pos * HK * D, kb, (size_t)HK * D * sizeof(float));
        memcpy(vl + pos * HK * D, v + (size_t)b * HK * D, (size_t)HK * D * sizeof(float));
        #pragma omp parallel for schedule(static)
        for (int h = 0; h < H; h++) {
            float* scores = (float*)malloc(n * sizeof(float));
            if (!scores) { err = 1; continue; }
            int kvh = h * HK / H;
            head_attend(qb + (size_t)h * D, kl + (size_t)kvh * D, vl + (size_t)kvh * D,
                        (size_t)HK * D, n, D, scale, scores, ao + ((size_t)b * H + h) * D);
            free(scores);
        }
    }
    return err ? ORACLE_ERR_MEMORY : ORACLE_OK;
}

/* Attention only (no RoPE, no append) of already-rotated queries
 * q [H][D] over a pos-major cache region of n rows; used to check
 * partial/sharded results against whole-cache attention. */
int oracle_attend_rows(int H, int HK, int D, size_t n, const float* kc, const float* vc,
                       const float* q, float* ao) {
    if (n == 0 || H % HK) return ORACLE_ERR_ARG;
    const float scale = 1.0f / sqrtf((float)D);
    int err = 0;
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++) {
        float* scores = (float*)malloc(n * sizeof(float));
        if (!scores) { err = 1; continue; }
        int kvh = h * HK / H;
        head_attend(q + (size_t)h * D, kc + (size_t)kvh * D, vc + (size_t)kvh * D,
                    (size_t)HK * D, n, D, scale, scores, ao + (size_t)h * D);
        free(scores);
    }
    return err ? ORACLE_ERR_MEMORY : ORACLE_OK;
}

/* Rotate x [n_heads][D] in place with table row `pos`; exposed so the
 * tests can build rotated inputs for the sharded checks. */
void oracle_rope_apply(float* x, int n_heads, int D, const float* sin_row, const float* cos_row) {
    int half = D / 2 > 64 ? 64 : D / 2;
    rope_rotate(x, n_heads, D, half, sin_row, cos_row);
}
