// decode_splitkv.cuh - split-KV flash-decoding for pickle's GQA attention
// block on sm_100a (RoPE + KV append + attention + split combine in one
// launch).
//
// Replaces lee-muriithi-kingori/lestramanika src/pickle_fast.c:1910-2094
// for decode: RoPE on q and the new k (:1913-1936), the cache append
// (:1939-1944), scores scaled by 1/sqrtf(D) (:1958-2032), softmax
// (:2034-2044) and the weighted sum of V (:2046-2091), for every query
// head h with kv_head = h * HK / H (:1963).
//
// Work decomposition. One CTA owns (split, kv_head, query z) and streams a
// contiguous run of cache rows of that KV head: in the head-major layout
// [seq][kv_head][pos][D] the run is one contiguous byte range, so each tile
// of TP=32 rows of K (and of V) is a single 1-D bulk TMA copy into a
// STAGES-deep shared-memory ring guarded by mbarriers. One producer lane
// issues the copies; G consumer warps (G = H / HK query heads share each
// KV head, so K/V are read from HBM once per KV head, not once per query
// head as the reference's loop does) each take 32/G rows of every tile.
// A lane holds a float4 slice of every query head in registers, the
// per-row partial dots of all (row, head) pairs of the warp are summed by
// a 5-level reduce-scatter (31 shuffles for 32 dot products), the online
// softmax keeps a running (max, sum) per head and rescales the float4
// accumulators, and P.V reuses the same float4 slices of V.
//
// The new token's row (RoPE'd k, v) is stored to the cache and attended
// from shared memory by the CTA of the last split, so no CTA ever reads a
// row another CTA of the same launch writes. With one split a CTA writes
// the normalised output itself. With several, each CTA publishes its
// unnormalised partial (m, l, acc) and decode_merge_kernel combines them:
// it is launched as a programmatic dependent of the split kernel, so its
// CTAs are resident before the split kernel retires and start merging as
// soon as the partials are visible. Spreading the merge over one CTA per
// output row keeps it off a single SM's L2 bandwidth (a merge by the last
// split CTA of each group, which pulls the group's partials through one
// SM, measured 2-4 us slower a step at B=1 and B=8).
//
// The split kernel itself waits in griddepcontrol.wait before its first
// global access, so it can be launched as a programmatic dependent of the
// kernel before it on the stream (the previous decode step, or the
// projection that wrote q / k / v): its CTAs become resident while that
// kernel's last CTAs run.
#pragma once
#include <cfloat>
#include <cmath>
#include "pcu_common.cuh"

struct DecodeArgs {
    const float* q;          // [n_z][H][D], z = seq * n_q + t
    const float* k_new;      // [n_seqs][HK][D] (append)
    const float* v_new;
    float* kc;               // this layer's K cache
    float* vc;
    long long seq_stride;    // floats between sequences in the cache
    long long head_stride;   // floats between KV heads (= max_seq * D)
    const float* sin_tab;    // [max_seq][half]
    const float* cos_tab;
    int H, HK, half;
    int n_q;                 // queries per sequence in this launch
    long long q_pos0;        // absolute position of query t = 0 (RoPE row)
    int rope;                // rotate q and k_new with the table row at the query position
    int vec;                 // half % 4 == 0 and 16-byte aligned tables: float4 RoPE loads
    int append;              // store + attend the new k/v row
    long long append_idx;    // cache row of the new token
    long long hist_len0;     // cached rows [0, hist) attended by query t = 0
    int hist_step;           // query t attends hist_len0 + t * hist_step rows
    int n_splits;
    int l2_ahead;            // short splits: tiles requested into L2 beyond the shared-memory copies
    int early_l2;            // tiles of the split requested into L2 before griddepcontrol.wait (0: none)
    long long chunk;         // history rows per split
    float scale;             // 1 / sqrtf(D)
    int out_mode;            // 0: ao = normalised output; 1: unnormalised (m, l, acc)
    int force_partials;      // write split partials to ws_* even with one split (a merge kernel follows)
    float* ao;               // [n_z][H][D]
    float* out_m;            // [n_z][H] (out_mode 1)
    float* out_l;
    float* ws_m;             // [n_groups][G][n_splits]
    float* ws_l;
    float* ws_acc;           // [n_groups][G][n_splits][D]
    int* err;
    // Ragged decode (continuous batching), else null: entry z attends its
    // own seq_pos[z] cached rows, rotates with and appends at that position,
    // in cache slot seq_slot[z] (null: slot z). Positions above max_pos and
    // slots outside [0, n_slots) are rejected on the device (error word).
    const int* seq_pos;
    const int* seq_slot;
    long long max_pos;
    int n_slots;
};

constexpr int kMaxSplits = 256;
// Tiles a short split (one that staggers its first tile) keeps requested
// into L2 beyond its shared-memory ring. Measured on B200: +6 % at B=1
// (3.5 tiles per split); streaming splits lose 4-30 % with any look-ahead
// (the extra L2 traffic competes with the ring's own copies), so they
// take none.
constexpr int kDefaultL2Ahead = 2;

// Host: the split count for `groups` independent (query, KV head) streams
// of `hist` cached rows of D floats, on `slots` resident CTA slots, among
// split counts 1..max_s that cut hist into exactly that many pieces. A
// plan's estimated time: each wave of CTAs streams its K/V chunk at
// min(one CTA's rate, HBM bandwidth / CTAs in the wave), each wave costs a
// fixed ramp, and several splits add the merge launch. One CTA (two per SM,
// eight consumer warps) streams at most ~33 GB/s with four query heads per
// KV head and ~22 GB/s with eight (issue-bound), so a partial last wave
// runs at that rate alone, while one wave of fewer CTAs than slots can
// still fill HBM. The constants were fitted on B200 to split-count sweeps
// of six decode shapes (GQA 4: B=1/8/64 at ctx 4096, B=1 at ctx 131072;
// GQA 8: B=2 and B=16 at ctx 32768); in each the plan below picks the
// measured fastest count.
inline double decode_plan_time(long long groups, long long hist, long long slots, long long s, int G, int D) {
    const double hbm = 6.5e12;                          // bytes/s
    const double cta_rate = G > 4 ? 22e9 : 33e9;        // bytes/s of one CTA
    const double wave_cost = 3e-6, merge_cost = 4e-6;   // seconds
    const long long chunk = (hist + s - 1) / s;
    const long long n = groups * s, full = n / slots, rem = n % slots;
    const double bytes = (double)chunk * 2.0 * D * sizeof(float);
    const double full_rate = cta_rate < hbm / (double)slots ? cta_rate : hbm / (double)slots;
    double t = (double)full * bytes / full_rate;
    if (rem) {
        const double rem_rate = cta_rate < hbm / (double)rem ? cta_rate : hbm / (double)rem;
        t += bytes / rem_rate;
    }
    t += wave_cost * (double)(full + (rem ? 1 : 0));
    if (s > 1) t += merge_cost;
    return t;
}

// Among counts within 0.5 % of the fastest estimate, the most splits: where
// a wave saturates HBM either way, more CTAs hide more latency (measured:
// 37 splits over 30 at B=1, ctx 4096).
inline int plan_decode_splits(long long groups, long long hist, long long slots, long long max_s, int G, int D) {
    if (hist <= 0 || groups <= 0 || slots <= 0) return 1;
    if (max_s < 1) max_s = 1;
    auto exact = [&](long long s) { const long long c = (hist + s - 1) / s; return (hist + c - 1) / c == s; };
    double best_t = -1.0;
    for (long long s = 1; s <= max_s; ++s) {
        if (!exact(s)) continue;
        const double t = decode_plan_time(groups, hist, slots, s, G, D);
        if (best_t < 0 || t < best_t) best_t = t;
    }
    int best = 1;
    for (long long s = 1; s <= max_s; ++s)
        if (exact(s) && decode_plan_time(groups, hist, slots, s, G, D) <= best_t * 1.005) best = (int)s;
    return best;
}

template <int D, int G>
struct DecodeCfg {
    static constexpr int GS = G > 4 ? 4 : G;      // query heads per warp
    static constexpr int NHG = G / GS;            // head groups (warps of a group split the tile's rows)
    static constexpr int NW = G;                  // warps of a consumer set = NHG groups x GS warps
    static constexpr int RPW = 32 / GS;           // rows per warp per tile
    static constexpr int TP = 32;                 // rows per tile
    static constexpr int NCH = D / 4;             // float4 chunks per row
    static constexpr int CPL = (NCH + 31) / 32;   // chunks per lane
    static constexpr int ROW_BYTES = D * 4;
    static constexpr int TILE_BYTES = TP * ROW_BYTES;
    static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
    static constexpr int STAGES_RAW = 98304 / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
    // Consumer sets: set k takes tiles k, k + NSET, ... with its own online
    // softmax state, so up to eight consumer warps (four for D > 128, whose
    // query and accumulator slices take twice the registers) share one
    // CTA's ring, never more sets than tiles in flight.
    static constexpr int NSET_RAW = (D > 128 ? 4 : 8) / G;
    static constexpr int NSET = NSET_RAW < 1 ? 1 : (NSET_RAW > STAGES ? STAGES : NSET_RAW);
    static constexpr int NCW = NSET * NW;         // consumer warps
    static constexpr int WPH = NSET * GS;         // warps holding partial state of one query head
    static constexpr int THREADS = (NCW + 1) * 32;
    static constexpr int MIN_CTAS = 2;            // two CTAs per SM
    static constexpr size_t RING_BYTES = (size_t)STAGES * STAGE_BYTES;
    static constexpr size_t NEWROW_OFF = RING_BYTES;
    static constexpr size_t PBUF_OFF = NEWROW_OFF + 2 * ROW_BYTES;
    static constexpr size_t BAR_OFF = (PBUF_OFF + NCW * 32 * 4 + 15) / 16 * 16;
    static constexpr size_t SMEM = BAR_OFF + 2 * STAGES * 8;
    // Epilogue scratch reuses the ring: the per-warp (acc, m, l) of the
    // intra-CTA merge.
    static constexpr int RING_FLOATS = (int)(RING_BYTES / 4);
    static constexpr int INTRA = NCW * GS * D + 2 * NCW * GS;
    static_assert(D % 4 == 0, "rows must be 16-byte multiples");
    static_assert(32 % G == 0 && G <= 8, "G in {1, 2, 4, 8}");
    static_assert(INTRA <= RING_FLOATS, "epilogue scratch must fit in the ring");
    static_assert(NSET >= 1 && THREADS <= 288, "at most eight consumer warps");
};

// NeoX rotation of element d of a head row x (src/pickle_fast.c:1917-1924).
PCU_DEV float rope_elem(const float* x, int d, int half, const float* sr, const float* cr) {
    if (d < half) {
        const float lo = x[d], hi = x[d + half];
        return cr[d] * lo - sr[d] * hi;
    }
    if (d < 2 * half) {
        const int i = d - half;
        const float lo = x[i], hi = x[d];
        return sr[i] * lo + cr[i] * hi;
    }
    return x[d];
}

PCU_DEV float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Elements 4c..4c+3 of a rotated head row with 16-byte loads: the same
// products and sums as rope_elem (needs half % 4 == 0 and aligned rows).
PCU_DEV float4 rope_vec4(const float* x, int c, int half, const float* sr, const float* cr) {
    const int d = 4 * c;
    if (d < half) {
        const float4 lo = ld4(x + d), hi = ld4(x + d + half), sn = ld4(sr + d), cs = ld4(cr + d);
        return make_float4(cs.x * lo.x - sn.x * hi.x, cs.y * lo.y - sn.y * hi.y,
                           cs.z * lo.z - sn.z * hi.z, cs.w * lo.w - sn.w * hi.w);
    }
    if (d < 2 * half) {
        const int i = d - half;
        const float4 lo = ld4(x + i), hi = ld4(x + d), sn = ld4(sr + i), cs = ld4(cr + i);
        return make_float4(sn.x * lo.x + cs.x * hi.x, sn.y * lo.y + cs.y * hi.y,
                           sn.z * lo.z + cs.z * hi.z, sn.w * lo.w + cs.w * hi.w);
    }
    return ld4(x + d);
}

// Chunk c of a head row, rotated (rope) or not.
PCU_DEV float4 load_row4(const float* x, int c, int rope, int vec, int half, const float* sr,
                         const float* cr) {
    if (!rope) return ld4(x + 4 * c);
    if (vec) return rope_vec4(x, c, half, sr, cr);
    return make_float4(rope_elem(x, 4 * c + 0, half, sr, cr), rope_elem(x, 4 * c + 1, half, sr, cr),
                       rope_elem(x, 4 * c + 2, half, sr, cr), rope_elem(x, 4 * c + 3, half, sr, cr));
}

// Two FP32 fused multiply-adds in one sm_100 instruction (fma.rn.f32x2):
// exactly the same rounding as two fmaf calls.
PCU_DEV float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

PCU_DEV float2 mul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// One reduce-scatter level: lanes exchange the half of their W+W values
// they do not keep; afterwards v[0..W) hold sums over lane pairs (l, l^W).
template <int W>
PCU_DEV void rs_level(float (&v)[32], int lane) {
    const bool up = (lane & W) != 0;
    #pragma unroll
    for (int i = 0; i < W; ++i) {
        const float send = up ? v[i] : v[i + W];
        const float keep = up ? v[i + W] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, W);
    }
}

// The same level when lane l's values are stored at index (value ^ l): every
// lane keeps its lower half and sends its upper half, with no selects.
template <int W>
PCU_DEV void rs_level_xor(float (&v)[32]) {
    #pragma unroll
    for (int i = 0; i < W; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i + W], W);
}

// After this, lane l holds the warp-wide sum of value index l. Value indices
// are row * GS + head; lane l stores the value of row r at index
// ((r ^ (l / GS)) * GS + head), so the row levels (W >= GS) run select-free.
template <int GS>
PCU_DEV float reduce_scatter32(float (&v)[32], int lane) {
    rs_level_xor<16>(v);
    if constexpr (GS <= 8) rs_level_xor<8>(v); else rs_level<8>(v, lane);
    if constexpr (GS <= 4) rs_level_xor<4>(v); else rs_level<4>(v, lane);
    if constexpr (GS <= 2) rs_level_xor<2>(v); else rs_level<2>(v, lane);
    if constexpr (GS <= 1) rs_level_xor<1>(v); else rs_level<1>(v, lane);
    return v[0];
}

// One warp attends `nvalid` (1..RPW) consecutive rows at Kw/Vw (shared
// memory, row stride D) and folds them into its running softmax state.
// FULL: all RPW rows are valid, so the row checks fold away (every tile
// but a split's last takes this path; without the checks the GQA-8
// kernel issues ~10 % fewer instructions a tile and streams 7 % faster).
template <int D, int G, bool FULL = false>
PCU_DEV void attend_rows(const float* __restrict__ Kw, const float* __restrict__ Vw, int nvalid_arg,
                         const float4 (&qr)[G][DecodeCfg<D, G>::CPL],
                         float4 (&acc)[G][DecodeCfg<D, G>::CPL], float& m_run, float& l_run,
                         float* pw, float scale, int lane) {
    using C = DecodeCfg<D, G>;
    const int nvalid = FULL ? C::RPW : nvalid_arg;
    float vals[32];
    const int rx = lane / G;                         // this lane's row permutation (reduce_scatter32)
    #pragma unroll
    for (int r = 0; r < C::RPW; ++r) {
        const int row = r ^ rx;                      // the row whose values go to index r * G + g
        float4 kr[C::CPL];
        #pragma unroll
        for (int i = 0; i < C::CPL; ++i) {
            const int c = lane + 32 * i;
            kr[i] = (row < nvalid && c < C::NCH) ? reinterpret_cast<const float4*>(Kw + row * D)[c]
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        #pragma unroll
        for (int g = 0; g < G; ++g) {
            float2 s2 = make_float2(0.f, 0.f);
            #pragma unroll
            for (int i = 0; i < C::CPL; ++i) {
                s2 = fma2(make_float2(qr[g][i].x, qr[g][i].y), make_float2(kr[i].x, kr[i].y), s2);
                s2 = fma2(make_float2(qr[g][i].z, qr[g][i].w), make_float2(kr[i].z, kr[i].w), s2);
            }
            vals[r * G + g] = s2.x + s2.y;
        }
    }
    float s = reduce_scatter32<G>(vals, lane);       // lane l: row l / G, head l % G
    s = (lane / G < nvalid) ? s * scale : -INFINITY;
    float tmax = s;
    #pragma unroll
    for (int m = G; m < 32; m <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, m));
    const float m_new = fmaxf(m_run, tmax);
    const float p = expf(s - m_new);
    float psum = p;
    #pragma unroll
    for (int m = G; m < 32; m <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, m);
    // The sum and the accumulators are rescaled only when some head's running
    // maximum grew (after the first tiles it rarely does); otherwise the
    // factor is 1 and is skipped.
    if (__any_sync(0xffffffffu, m_new != m_run)) {
        const float alpha = expf(m_run - m_new);
        l_run = l_run * alpha + psum;
        #pragma unroll
        for (int g = 0; g < G; ++g) {
            const float ag = __shfl_sync(0xffffffffu, alpha, g);
            const float2 a2 = make_float2(ag, ag);
            #pragma unroll
            for (int i = 0; i < C::CPL; ++i) {
                const float2 lo = mul2(make_float2(acc[g][i].x, acc[g][i].y), a2);
                const float2 hi = mul2(make_float2(acc[g][i].z, acc[g][i].w), a2);
                acc[g][i] = make_float4(lo.x, lo.y, hi.x, hi.y);
            }
        }
    } else {
        l_run += psum;
    }
    m_run = m_new;
    pw[lane] = p;
    __syncwarp();
    #pragma unroll
    for (int r = 0; r < C::RPW; ++r) {
        if (r < nvalid) {
            float pr[G];
            if constexpr (G == 4) {         // one 16-byte shared load (pw rows are 16-byte aligned)
                const float4 p4 = *reinterpret_cast<const float4*>(pw + r * 4);
                pr[0] = p4.x; pr[1] = p4.y; pr[2] = p4.z; pr[3] = p4.w;
            } else {
                #pragma unroll
                for (int g = 0; g < G; ++g) pr[g] = pw[r * G + g];
            }
            #pragma unroll
            for (int i = 0; i < C::CPL; ++i) {
                const int c = lane + 32 * i;
                if (c < C::NCH) {
                    const float4 vv = reinterpret_cast<const float4*>(Vw + r * D)[c];
                    #pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float2 pp = make_float2(pr[g], pr[g]);
                        const float2 lo = fma2(pp, make_float2(vv.x, vv.y), make_float2(acc[g][i].x, acc[g][i].y));
                        const float2 hi = fma2(pp, make_float2(vv.z, vv.w), make_float2(acc[g][i].z, acc[g][i].w));
                        acc[g][i] = make_float4(lo.x, lo.y, hi.x, hi.y);
                    }
                }
            }
        }
    }
    __syncwarp();
}

// L2 prefetch of the K and V tiles [t0, t1) of a split of n_rows rows.
template <class C>
PCU_DEV void prefetch_l2_tiles(const float* kbase, const float* vbase, int n_rows, int t0, int t1) {
    for (int it = t0; it < t1; ++it) {
        const int rows = min(C::TP, n_rows - it * C::TP);
        const uint32_t bytes = (uint32_t)rows * C::ROW_BYTES;
        bulk_prefetch_l2(kbase + (size_t)it * C::TP * (C::ROW_BYTES / 4), bytes);
        bulk_prefetch_l2(vbase + (size_t)it * C::TP * (C::ROW_BYTES / 4), bytes);
    }
}

template <int D, int G>
__global__ void __launch_bounds__(DecodeCfg<D, G>::THREADS, DecodeCfg<D, G>::MIN_CTAS)
decode_splitkv_kernel(const DecodeArgs a) {
    using C = DecodeCfg<D, G>;
    extern __shared__ __align__(128) unsigned char smem[];
    float* ring = reinterpret_cast<float*>(smem);
    float* newK = reinterpret_cast<float*>(smem + C::NEWROW_OFF);
    float* newV = newK + D;
    float* pbuf = reinterpret_cast<float*>(smem + C::PBUF_OFF);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty = full + C::STAGES;
    __shared__ int s_abort, s_issued;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z;
    // While the kernel before it finishes, the producer lane asks L2 for the
    // split's first cached rows. A prefetch only warms L2, which every write
    // reaches, so it cannot return stale data; the copies that read the rows
    // are issued after the wait. (Not for ragged batches: their positions are
    // in device memory the kernel before may write.)
    if (a.early_l2 > 0 && !a.seq_pos && warp == C::NCW && lane == 0) {
        const long long h0 = a.hist_len0 + (long long)(z % a.n_q) * a.hist_step;
        const long long r0 = (long long)split * a.chunk;
        const long long r1 = r0 + a.chunk < h0 ? r0 + a.chunk : h0;
        const int nr = r1 > r0 ? (int)(r1 - r0) : 0;
        const size_t off = (size_t)(z / a.n_q) * a.seq_stride + (size_t)kvh * a.head_stride + (size_t)r0 * D;
        prefetch_l2_tiles<C>(a.kc + off, a.vc + off, nr, 0, min((nr + C::TP - 1) / C::TP, a.early_l2));
    }
    // Launched as a programmatic dependent of the kernel before it on the
    // stream: nothing that kernel writes (q / k / v, the cache) is read
    // before it completes.
    griddep_wait();
    int seq = z / a.n_q;
    const int t = z % a.n_q;
    long long hist = a.hist_len0 + (long long)t * a.hist_step;
    long long chunk = a.chunk, qpos = a.q_pos0 + t, append_idx = a.append_idx;
    if (a.seq_pos) {
        const long long p = a.seq_pos[z];
        if (a.seq_slot) seq = a.seq_slot[z];
        if (p < 0 || p > a.max_pos || seq < 0 || seq >= a.n_slots) {
            if (tid_is_first()) record_error(a.err, PCU_DEVERR_ARG);
            return;
        }
        hist = qpos = append_idx = p;
        chunk = p > 0 ? (p + a.n_splits - 1) / a.n_splits : 1;
    }
    const long long row0 = (long long)split * chunk;
    long long row1 = row0 + chunk;
    if (row1 > hist) row1 = hist;
    const int n_rows = row1 > row0 ? (int)(row1 - row0) : 0;
    const bool do_append = a.append && split == a.n_splits - 1;
    const size_t head_off = (size_t)seq * a.seq_stride + (size_t)kvh * a.head_stride;
    const float* kbase = a.kc + head_off + (size_t)row0 * D;
    const float* vbase = a.vc + head_off + (size_t)row0 * D;
    const int n_tiles = (n_rows + C::TP - 1) / C::TP;
    // A short split (small batches, where every CTA starts at once) puts only
    // its first tile in flight and requests the other stages once it lands:
    // the first tiles then arrive early and compute overlaps the rest of the
    // stream, instead of every CTA's tiles arriving interleaved at the end.
    const bool stagger = n_tiles <= 2 * C::STAGES;
    const int l2_ahead = stagger ? a.l2_ahead : 0;
    const float* sr = a.sin_tab + (size_t)qpos * a.half;
    const float* cr = a.cos_tab + (size_t)qpos * a.half;

    float4 acc[C::GS][C::CPL];
    float4 qr[C::GS][C::CPL];
    float m_run = -INFINITY, l_run = 0.f;
    int first_issued = 0;

    griddep_launch_dependents();                        // the next kernel's CTAs may take free SM slots now

    // Prologue. The producer lane sets up the ring and puts the first
    // STAGES tile copies in flight at once; meanwhile the consumer warps
    // rotate and store the new row (last split) and load their query heads.
    if (warp == C::NCW) {
        if (lane == 0) {
            for (int s = 0; s < C::STAGES; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], C::NW);
            }
            mbar_fence_init();
            s_abort = 0;
            s_issued = 0;
            first_issued = n_tiles < C::STAGES ? n_tiles : C::STAGES;
            if (stagger && first_issued > 1) first_issued = 1;
            for (int it = 0; it < first_issued; ++it) {
                const int rows = min(C::TP, n_rows - it * C::TP);
                const uint32_t bytes = (uint32_t)rows * C::ROW_BYTES;
                float* ks = ring + (size_t)it * (C::STAGE_BYTES / 4);
                mbar_arrive_expect_tx(&full[it], 2u * bytes);
                bulk_g2s(ks, kbase + (size_t)it * C::TP * D, bytes, &full[it]);
                bulk_g2s(ks + C::TILE_BYTES / 4, vbase + (size_t)it * C::TP * D, bytes, &full[it]);
            }
            // The next l2_ahead tiles go to L2 at once: a split's DRAM requests
            // are then in flight from the start instead of one ring's worth.
            prefetch_l2_tiles<C>(kbase, vbase, n_rows, first_issued, min(n_tiles, first_issued + l2_ahead));
        }
    } else {
        if (do_append) {
            const float* kn = a.k_new + ((size_t)z * a.HK + kvh) * D;
            const float* vn = a.v_new + ((size_t)z * a.HK + kvh) * D;
            float4* kdst = reinterpret_cast<float4*>(a.kc + head_off + (size_t)append_idx * D);
            float4* vdst = reinterpret_cast<float4*>(a.vc + head_off + (size_t)append_idx * D);
            for (int c = tid; c < C::NCH; c += C::NCW * 32) {
                const float4 kk = load_row4(kn, c, a.rope, a.vec, a.half, sr, cr);
                const float4 vv = ld4(vn + 4 * c);
                reinterpret_cast<float4*>(newK)[c] = kk;
                reinterpret_cast<float4*>(newV)[c] = vv;
                kdst[c] = kk;
                vdst[c] = vv;
            }
        }
        // Warp w serves head group hg = (w % NW) / GS: GS query heads of this KV head.
        const int hg = (warp % C::NW) / C::GS;
        const float* qh0 = a.q + ((size_t)z * a.H + (size_t)kvh * G + hg * C::GS) * D;
        #pragma unroll
        for (int g = 0; g < C::GS; ++g) {
            #pragma unroll
            for (int i = 0; i < C::CPL; ++i) {
                const int c = lane + 32 * i;
                qr[g][i] = c < C::NCH ? load_row4(qh0 + (size_t)g * D, c, a.rope, a.vec, a.half, sr, cr)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                acc[g][i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    __syncthreads();

    if (warp == C::NCW) {
        // Producer: one lane streams the K/V tiles of this split.
        if (lane == 0) {
            int issued = first_issued;
            for (int it = first_issued; it < n_tiles; ++it) {
                const int s = it % C::STAGES;
                if (stagger && it == 1 && !mbar_wait(&full[0], 0)) {
                    record_error(a.err, PCU_DEVERR_EMPTY_WAIT);
                    s_abort = 1;
                    break;
                }
                if (it >= C::STAGES && !mbar_wait(&empty[s], ((it / C::STAGES) - 1) & 1)) {
                    record_error(a.err, PCU_DEVERR_EMPTY_WAIT);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int*)&s_abort) break;
                const int rows = min(C::TP, n_rows - it * C::TP);
                const uint32_t bytes = (uint32_t)rows * C::ROW_BYTES;
                float* ks = ring + (size_t)s * (C::STAGE_BYTES / 4);
                float* vs = ks + C::TILE_BYTES / 4;
                mbar_arrive_expect_tx(&full[s], 2u * bytes);
                bulk_g2s(ks, kbase + (size_t)it * C::TP * D, bytes, &full[s]);
                bulk_g2s(vs, vbase + (size_t)it * C::TP * D, bytes, &full[s]);
                issued = it + 1;
                // Keep tiles [issued, issued + l2_ahead) requested: the tile
                // entering that window now has not been requested before.
                const int pf = it + l2_ahead;
                if (l2_ahead > 0 && pf >= first_issued + l2_ahead && pf < n_tiles)
                    prefetch_l2_tiles<C>(kbase, vbase, n_rows, pf, pf + 1);
            }
            s_issued = issued;
        }
    } else {
        // Consumers: warp w belongs to set w / NW, which takes tiles set,
        // set + NSET, ...; within the set it serves head group (w % NW) / GS
        // and rows [wi * RPW, (wi + 1) * RPW) of each of its tiles.
        constexpr int GS = C::GS;
        const int set = warp / C::NW, wi = (warp % C::NW) % GS;
        float* pw = pbuf + warp * 32;
        for (int it = set; it < n_tiles; it += C::NSET) {
            const int s = it % C::STAGES;
            if (C::NSET > 1 && it >= C::STAGES) {
                // Consecutive uses of a stage may belong to different sets. Wait
                // for the release of the previous use (tile it - STAGES) first:
                // then the stage's full barrier is at most one phase away and
                // its parity wait cannot match the phase two uses back.
                const bool rel = __all_sync(0xffffffffu, mbar_wait(&empty[s], ((it / C::STAGES) - 1) & 1));
                if (!rel) {
                    if (lane == 0) { record_error(a.err, PCU_DEVERR_EMPTY_WAIT); s_abort = 1; }
                    break;
                }
            }
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / C::STAGES) & 1));
            if (!ok) {
                if (lane == 0) { record_error(a.err, PCU_DEVERR_FULL_WAIT); s_abort = 1; }
                break;
            }
            const int rows = min(C::TP, n_rows - it * C::TP);
            const int nvalid = min(max(rows - wi * C::RPW, 0), C::RPW);
            const float* ks = ring + (size_t)s * (C::STAGE_BYTES / 4);
            const float* vs = ks + C::TILE_BYTES / 4;
            if (nvalid == C::RPW)
                attend_rows<D, GS, true>(ks + wi * C::RPW * D, vs + wi * C::RPW * D, nvalid, qr, acc,
                                         m_run, l_run, pw, a.scale, lane);
            else if (nvalid > 0)
                attend_rows<D, GS>(ks + wi * C::RPW * D, vs + wi * C::RPW * D, nvalid, qr, acc,
                                   m_run, l_run, pw, a.scale, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (do_append && set == n_tiles % C::NSET && wi == 0 && !*(volatile int*)&s_abort)
            attend_rows<D, GS>(newK, newV, 1, qr, acc, m_run, l_run, pw, a.scale, lane);
    }
    __syncthreads();

    if (s_abort) {
        // Let the copies still in flight land before the CTA's shared memory goes away.
        if (tid == 0) {
            const int issued = s_issued;
            for (int it = issued > C::STAGES ? issued - C::STAGES : 0; it < issued; ++it)
                if (!mbar_wait(&full[it % C::STAGES], (it / C::STAGES) & 1))
                    record_error(a.err, PCU_DEVERR_DRAIN_WAIT);
        }
        return;
    }

    // ---- epilogue: merge the warps holding each query head's state ----
    constexpr int GS = C::GS;
    const size_t gidx = (size_t)z * a.HK + kvh;
    float* sm_acc = ring;                               // [NCW][GS][D]
    float* sm_m = sm_acc + C::NCW * GS * D;             // [NCW][GS]
    float* sm_l = sm_m + C::NCW * GS;                   // [NCW][GS]
    // Warp j (0 <= j < WPH) holding state of local head gl of head group hg.
    auto head_warp = [&](int hg, int j) { return (j / GS) * C::NW + hg * GS + j % GS; };

    if (warp < C::NCW) {
        if (lane < GS) {
            sm_m[warp * GS + lane] = m_run;
            sm_l[warp * GS + lane] = l_run;
        }
        #pragma unroll
        for (int g = 0; g < GS; ++g)
            #pragma unroll
            for (int i = 0; i < C::CPL; ++i) {
                const int c = lane + 32 * i;
                if (c < C::NCH) reinterpret_cast<float4*>(sm_acc + (warp * GS + g) * D)[c] = acc[g][i];
            }
    }
    __syncthreads();

    // Thread (g, c): weights of the WPH warps holding head g, computed by
    // every thread of the head (no second barrier), then chunk c of the
    // head's partial.
    for (int idx = tid; idx < G * C::NCH; idx += C::THREADS) {
        const int g = idx / C::NCH, c = idx % C::NCH, hg = g / GS, gl = g % GS;
        float mw[C::WPH];
        float M = -INFINITY;
        #pragma unroll
        for (int j = 0; j < C::WPH; ++j) {
            mw[j] = sm_m[head_warp(hg, j) * GS + gl];
            M = fmaxf(M, mw[j]);
        }
        float L = 0.f;
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
        #pragma unroll
        for (int j = 0; j < C::WPH; ++j) {
            const float e = (mw[j] == -INFINITY) ? 0.f : expf(mw[j] - M);
            L = fmaf(sm_l[head_warp(hg, j) * GS + gl], e, L);
            const float4 x = reinterpret_cast<const float4*>(sm_acc + (head_warp(hg, j) * GS + gl) * D)[c];
            A.x = fmaf(e, x.x, A.x); A.y = fmaf(e, x.y, A.y);
            A.z = fmaf(e, x.z, A.z); A.w = fmaf(e, x.w, A.w);
        }
        if (a.n_splits > 1 || a.force_partials) {
            // Partial of this split; decode_merge_kernel combines the splits.
            const size_t prow = (gidx * G + g) * a.n_splits + split;
            reinterpret_cast<float4*>(a.ws_acc + prow * D)[c] = A;
            if (c == 0) { a.ws_m[prow] = M; a.ws_l[prow] = L; }
            continue;
        }
        const size_t row = (size_t)z * a.H + (size_t)kvh * G + g;
        float4* dst = reinterpret_cast<float4*>(a.ao + row * D) + c;
        if (a.out_mode == 0) {
            const float inv = 1.0f / (L == 0.0f ? 1.0f : L);
            *dst = make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv);
        } else {
            *dst = A;
            if (c == 0) { a.out_m[row] = M; a.out_l[row] = L; }
        }
    }
}

// Combine the n_splits partials of every output row r (= z * H + h, which
// is also the partial row group (z * HK + kv_head) * G + local head):
//   M = max_s m_s, w_s = e^(m_s - M), L = sum_s w_s l_s,
//   out = sum_s w_s acc_s / L      (out_mode 1: sum_s w_s acc_s, M, L)
// i.e. the reference's softmax over all cached rows (src/pickle_fast.c
// :2034-2091) assembled from per-split maxima and sums. One CTA per row;
// thread (sg, c) takes float4 chunk c of splits sg, sg + SG, ... with all
// of its loads in flight, and the SG partial sums meet in shared memory.
struct MergeArgs {
    const float* ws_m;       // [n_rows][n_splits]
    const float* ws_l;
    const float* ws_acc;     // [n_rows][n_splits][D]
    int n_splits;
    int out_mode;
    float* out;              // [n_rows][D]
    float* out_m;            // [n_rows] (out_mode 1)
    float* out_l;
};

constexpr int kMergeThreads = 256;

template <int D>
struct MergeSmem {
    static constexpr int NCH = D / 4;
    static constexpr int SG = kMergeThreads / NCH;      // split groups
    float w[kMaxSplits];
    float M, L;
    float4 red[SG][NCH];
};

// The merge of one output row's split partials. Returns, in threads
// tid < D / 4, float4 chunk tid of the unnormalised sum_s w_s acc_s; sm.M
// and sm.L hold M and L. Thread (sg, c) takes chunk c of splits sg,
// sg + SG, ... with BATCH loads in flight. Ends with a CTA barrier.
template <int D>
PCU_DEV float4 merge_splits(const MergeArgs& a, int row, MergeSmem<D>& sm) {
    constexpr int NCH = D / 4;
    constexpr int SG = MergeSmem<D>::SG;
    constexpr int BATCH = 8;                            // loads in flight per thread per round
    const int tid = threadIdx.x;
    const int sg = tid / NCH, c = tid % NCH;
    const int S = a.n_splits;
    // Warp 0: split weights w_s = e^(m_s - M) into shared memory and L; the
    // other warps put their first batch of partial-row loads in flight.
    if (tid < 32) {
        constexpr int MS = kMaxSplits / 32;
        float mv[MS], lv[MS];
        #pragma unroll
        for (int j = 0; j < MS; ++j) {
            const int s = tid + 32 * j;
            mv[j] = s < S ? a.ws_m[(size_t)row * S + s] : -INFINITY;
            lv[j] = s < S ? a.ws_l[(size_t)row * S + s] : 0.f;
        }
        float M = -INFINITY;
        #pragma unroll
        for (int j = 0; j < MS; ++j) M = fmaxf(M, mv[j]);
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.f;
        #pragma unroll
        for (int j = 0; j < MS; ++j) {
            const int s = tid + 32 * j;
            const float e = (mv[j] == -INFINITY) ? 0.f : expf(mv[j] - M);
            if (s < S) sm.w[s] = e;
            L += lv[j] * e;
        }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (tid == 0) { sm.M = M; sm.L = L; }
    }
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4* src = reinterpret_cast<const float4*>(a.ws_acc + (size_t)row * S * D) + c;
    float4 x[BATCH];
    if (sg < SG) {
        #pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            const int s = sg + SG * j;
            x[j] = s < S ? src[(size_t)s * NCH] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    __syncthreads();
    if (sg < SG) {
        for (int s0 = sg; s0 < S; s0 += SG * BATCH) {
            if (s0 != sg) {
                #pragma unroll
                for (int j = 0; j < BATCH; ++j) {
                    const int s = s0 + SG * j;
                    x[j] = s < S ? src[(size_t)s * NCH] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            #pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                const int s = s0 + SG * j;
                if (s < S) {
                    const float e = sm.w[s];
                    A.x = fmaf(e, x[j].x, A.x); A.y = fmaf(e, x[j].y, A.y);
                    A.z = fmaf(e, x[j].z, A.z); A.w = fmaf(e, x[j].w, A.w);
                }
            }
        }
        sm.red[sg][c] = A;
    }
    __syncthreads();
    float4 T = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < NCH) {
        T = sm.red[0][tid];
        #pragma unroll
        for (int k = 1; k < SG; ++k) {
            const float4 y = sm.red[k][tid];
            T.x += y.x; T.y += y.y; T.z += y.z; T.w += y.w;
        }
    }
    return T;
}

template <int D>
__global__ void __launch_bounds__(kMergeThreads) decode_merge_kernel(const MergeArgs a) {
    __shared__ MergeSmem<D> sm;
    const int tid = threadIdx.x, row = blockIdx.x;
    griddep_launch_dependents();                        // the next decode step's CTAs may become resident
    griddep_wait();                                     // the split kernel's partials are visible
    const float4 T = merge_splits<D>(a, row, sm);
    if (tid < D / 4) {
        float4* dst = reinterpret_cast<float4*>(a.out + (size_t)row * D) + tid;
        if (a.out_mode == 0) {
            const float inv = 1.0f / (sm.L == 0.0f ? 1.0f : sm.L);
            *dst = make_float4(T.x * inv, T.y * inv, T.z * inv, T.w * inv);
        } else {
            *dst = T;
            if (tid == 0) { a.out_m[row] = sm.M; a.out_l[row] = sm.L; }
        }
    }
}

// Host: the merge launch, as a programmatic dependent of the split kernel
// just queued on `st` (its CTAs may become resident before the split
// kernel ends; griddepcontrol.wait holds them until the partials are
// visible). n_rows = queries x query heads.
inline cudaError_t launch_decode_merge(int D, const MergeArgs& m, int n_rows, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_rows);
    cfg.blockDim = dim3(kMergeThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (D) {
        case 48: return cudaLaunchKernelEx(&cfg, decode_merge_kernel<48>, m);
        case 64: return cudaLaunchKernelEx(&cfg, decode_merge_kernel<64>, m);
        case 96: return cudaLaunchKernelEx(&cfg, decode_merge_kernel<96>, m);
        case 128: return cudaLaunchKernelEx(&cfg, decode_merge_kernel<128>, m);
        case 256: return cudaLaunchKernelEx(&cfg, decode_merge_kernel<256>, m);
        default: return cudaErrorInvalidValue;
    }
}
