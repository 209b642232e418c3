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
// Work item: two 128-row query tiles (A = rows q0..q0+127, B = the next
// 128) of one (sequence, head); both share every K/V tile. The kernel is
// persistent: one CTA per SM takes items from a shared counter (heaviest
// first: every head's latest query block of a sequence, then the next
// lighter ones), and one item's tail overlaps the next item's start.
//   warp 8      one lane takes the next item, loads Q_A, Q_B (once the last
//               QK^T MMA of the previous item has read them) and streams K/V
//               tiles (128 keys) through a 2-stage ring with 3-D TMA tensor
//               copies (128-byte swizzle, no multicast);
//   warp 9      allocates 512 TMEM columns once - S_A, S_B, O_A, O_B, 128
//               each - and one lane issues tcgen05.mma in the order
//               PV_A(j), S_A(j+1), PV_B(j), S_B(j+1): S_X = Q_X K^T (both
//               operands in shared memory), O_X += P_X V (P_X read from TMEM,
//               V read MN-major from shared memory). An item's first PV_X
//               waits until the previous item's O_X has been read out;
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B: thread r
//               owns query row r (TMEM lane r). It loads its S row
//               (tcgen05.ld), masks, keeps the running max in the log2
//               domain (rescaling its O row in TMEM only when the max grows by
//               more than 2^8), writes P as packed BF16 over the first 64
//               columns of its S row (tcgen05.st) in two halves, keys 0-63
//               then 64-127, arriving on P_FULL_X after the first and P_HI_X
//               after the second: the MMA warp issues the first half of
//               P V while the second half is computed. At the item's end it reads
//               its O row, releases O_X and writes the normalised rows out
//               with TMA tensor stores (32 rows x 32 columns per store,
//               through a 4 KB per-warp shared-memory stage).
// MMAs issued by one thread execute in order, so S_FULL_X(j) also means
// PV_X(j-1) is complete (O_X may be rescaled), and S_X(j+1) cannot overwrite
// P_X(j) before PV_X(j) has read it. While one tile's softmax runs, the
// tensor core works on the other tile's MMAs.
// Every mbarrier wait is bounded; a timeout sets the error word, drains the
// copies and MMAs in flight, frees TMEM and exits.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>

#include "pcu_common.cuh"

namespace tc {

constexpr int BM = 128;                    // query rows per tile (two tiles per CTA)
constexpr int BN = 128;                    // keys per tile
constexpr int HD = 128;                    // head dim handled here
constexpr int HALF_BYTES = 128 * 128;      // one 64-column half of a 128-row tile (bf16)
constexpr int TILE_BYTES = 2 * HALF_BYTES; // 128 x 128 bf16
constexpr int STAGES = 2;
constexpr int SMEM_Q = 0;                                    // Q_A, Q_B
constexpr int SMEM_KV = SMEM_Q + 2 * TILE_BYTES;             // stage s: K at +2s*TILE, V at +(2s+1)*TILE
constexpr int SMEM_OUT = SMEM_KV + STAGES * 2 * TILE_BYTES;  // per softmax warp: 32 rows x 32 floats
constexpr int OUT_STAGE_BYTES = 32 * 32 * 4;
constexpr int SMEM_BAR = SMEM_OUT + 8 * OUT_STAGE_BYTES;
constexpr int N_BARS = 22;
constexpr int SMEM_BYTES = SMEM_BAR + N_BARS * 8 + 16 + 1024; // + TMEM address slot + alignment slack
static_assert(SMEM_BYTES <= 232448, "dynamic shared memory of one CTA on sm_100");
constexpr int WARP_TMA = 8, WARP_MMA = 9;
constexpr int THREADS = 320;
constexpr uint32_t TMEM_COLS = 512;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

// Barrier slots (+x: tile A / B, +s: ring stage, +i: item slot).
enum { B_Q_FULL = 0, B_Q_FREE = 1, B_KV_FULL = 2, B_KV_EMPTY = 4, B_S_FULL = 6, B_P_FULL = 8, B_O_DONE = 10,
       B_O_FREE = 12, B_ITEM_FULL = 14, B_ITEM_EMPTY = 16, B_DRAIN = 18, B_P_HI = 20 };
constexpr int SOFTMAX_WARPS = 8;

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

// TMA tensor store of one box from shared memory (bulk async group; rows
// past the tensor's bounds are not written).
PCU_DEV void tma_store_4d(uint32_t src, const CUtensorMap* map, int x, int y, int z, int w) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(src) : "memory");
}
PCU_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's committed stores have finished reading shared memory.
PCU_DEV void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// This thread's committed stores are complete.
PCU_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Generic-proxy writes to shared memory become visible to the TMA (async proxy).
PCU_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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

// D (TMEM) += A (TMEM, K-major, two BF16 per column) x B (shared memory).
PCU_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

PCU_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

PCU_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PCU_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

// TMEM lane loads/stores of 128 and 64 32-bit columns (generated).
PCU_DEV void tmem_ld128(uint32_t taddr, float (&v)[128]) {
    uint32_t r[128];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr)
        : "memory");
    #pragma unroll
    for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

PCU_DEV void tmem_st64(uint32_t taddr, const uint32_t (&v)[64]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};"
        :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]), "r"(v[32]), "r"(v[33]), "r"(v[34]), "r"(v[35]), "r"(v[36]), "r"(v[37]), "r"(v[38]), "r"(v[39]), "r"(v[40]), "r"(v[41]), "r"(v[42]), "r"(v[43]), "r"(v[44]), "r"(v[45]), "r"(v[46]), "r"(v[47]), "r"(v[48]), "r"(v[49]), "r"(v[50]), "r"(v[51]), "r"(v[52]), "r"(v[53]), "r"(v[54]), "r"(v[55]), "r"(v[56]), "r"(v[57]), "r"(v[58]), "r"(v[59]), "r"(v[60]), "r"(v[61]), "r"(v[62]), "r"(v[63])
        : "memory");
}

PCU_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x with one MUFU instruction (relative error ~2^-22, far below BF16 P).
PCU_DEV float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one sm_100 instruction (three-input max.f32).
PCU_DEV float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Two FP32 operations per instruction (sm_100 f32x2): same rounding as two
// scalar fmaf / additions.
PCU_DEV float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

PCU_DEV float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

PCU_DEV uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

struct PrefillTcArgs {
    float* ao;            // [n_seqs][T][H][D] F32
    int T, H, HK, n_qb;   // n_qb = query blocks of 2 * BM rows
    int n_seqs;
    int n_items;          // n_seqs * n_qb * H
    float scale_log2;     // log2(e) / sqrtf(D)
    unsigned* next_item;  // zero between launches; the last CTA to take from it resets it
    int* err;
};

struct PrefillItem {
    int h, seq, q0, n_kv_A, n_kv_B;
};

// Item i: head fastest, then query blocks latest (heaviest) first, then sequences.
PCU_DEV PrefillItem prefill_item(int i, const PrefillTcArgs& a) {
    PrefillItem it;
    it.h = i % a.H;
    const int r = i / a.H;
    const int qb = a.n_qb - 1 - r % a.n_qb;
    it.seq = r / a.n_qb;
    it.q0 = qb * 2 * BM;
    const int kv_tiles_T = (a.T + BN - 1) / BN;
    it.n_kv_A = min(it.q0 / BN + 1, kv_tiles_T);
    it.n_kv_B = min((it.q0 + BM) / BN + 1, kv_tiles_T);
    return it;
}

// S_X = Q_X K_j^T: M=128, N=128, K=HD in steps of 16 (32 bytes of a 128-byte swizzle row).
PCU_DEV void issue_qk(uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr) {
    const uint32_t id = idesc_bf16(BN, 0);
    #pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
        const uint32_t off = (ks / 4) * HALF_BYTES + (ks % 4) * 32;
        mma_bf16(d_tmem, smem_desc(q_addr + off, 16, 1024), smem_desc(k_addr + off, 16, 1024), id, ks > 0);
    }
}

// O_X += P_X V_j: A = P_X in TMEM (16 keys = 8 columns per step), B = V_j MN-major.
PCU_DEV void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_addr, bool first, int ks0, int ks1) {
    const uint32_t id = idesc_bf16(HD, 1);
    #pragma unroll
    for (int ks = ks0; ks < ks1; ++ks)
        mma_bf16_ts(o_tmem, p_tmem + ks * 8, smem_desc(v_addr + ks * 16 * 128, HALF_BYTES, 1024), id,
                    (!first || ks > 0));
}

__global__ void __launch_bounds__(THREADS, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const PrefillTcArgs a) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned base (128-byte swizzle atoms).
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_u32 - raw_u32);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + SMEM_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + SMEM_BAR + N_BARS * 8);
    __shared__ int s_abort, s_kv_issued, s_q_issued;
    __shared__ int s_item[2];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        mbar_init(&bars[B_Q_FULL], 1);
        mbar_init(&bars[B_Q_FREE], 1);
        for (int x = 0; x < 2; ++x) {
            mbar_init(&bars[B_KV_FULL + x], 1);
            mbar_init(&bars[B_KV_EMPTY + x], 1);
            mbar_init(&bars[B_S_FULL + x], 1);
            mbar_init(&bars[B_P_FULL + x], 4);
            mbar_init(&bars[B_P_HI + x], 4);
            mbar_init(&bars[B_O_DONE + x], 1);
            mbar_init(&bars[B_O_FREE + x], 4);
            mbar_init(&bars[B_ITEM_FULL + x], 1);
            mbar_init(&bars[B_ITEM_EMPTY + x], 1 + SOFTMAX_WARPS);
        }
        mbar_init(&bars[B_DRAIN], 1);
        mbar_fence_init();
        s_abort = 0;
        s_kv_issued = 0;
        s_q_issued = 0;
    }
    if (warp == WARP_MMA) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Launched as a programmatic dependent of the producer: the set-up above
    // overlaps its last CTAs; its q / k / v copies are read only after it ends.
    griddep_wait();
    const uint32_t tmem = *tmem_slot;
    auto aborted = [&]() { return *(volatile int*)&s_abort != 0; };
    auto fail = [&](int code) { record_error(a.err, code); s_abort = 1; };

    if (warp == WARP_TMA) {
        // ---------------- items, Q and the K/V ring ----------------
        if (lane == 0) {
            int g = 0;                                  // K/V tiles issued so far
            for (int k = 0;; ++k) {
                const int slot = k & 1;
                if (k >= 2 && !mbar_wait(&bars[B_ITEM_EMPTY + slot], ((k >> 1) - 1) & 1)) { fail(PCU_DEVERR_EMPTY_WAIT); break; }
                if (aborted()) break;
                const unsigned idx = atomicAdd(a.next_item, 1u);
                // Every CTA takes exactly one index past the end: the last of those resets the counter.
                if (idx == (unsigned)a.n_items + gridDim.x - 1u) *a.next_item = 0u;
                s_item[slot] = idx < (unsigned)a.n_items ? (int)idx : -1;
                mbar_arrive(&bars[B_ITEM_FULL + slot]);
                if (idx >= (unsigned)a.n_items) break;
                const PrefillItem it = prefill_item((int)idx, a);
                const int kvh = it.h * a.HK / a.H;     // src/pickle_fast.c:1963
                const int zq = it.seq * a.H + it.h, zk = it.seq * a.HK + kvh;
                // Q_A, Q_B may be overwritten once the previous item's last QK^T MMA has completed.
                if (k >= 1 && !mbar_wait(&bars[B_Q_FREE], (k - 1) & 1)) { fail(PCU_DEVERR_EMPTY_WAIT); break; }
                mbar_arrive_expect_tx(&bars[B_Q_FULL], 2 * TILE_BYTES);
                for (int x = 0; x < 2; ++x) {
                    tma_load_3d(base_u32 + SMEM_Q + x * TILE_BYTES, &tm_q, 0, it.q0 + x * BM, zq, &bars[B_Q_FULL]);
                    tma_load_3d(base_u32 + SMEM_Q + x * TILE_BYTES + HALF_BYTES, &tm_q, 64, it.q0 + x * BM, zq,
                                &bars[B_Q_FULL]);
                }
                s_q_issued = k + 1;
                for (int j = 0; j < it.n_kv_B; ++j, ++g) {
                    const int s = g % STAGES;
                    if (g >= STAGES && !mbar_wait(&bars[B_KV_EMPTY + s], ((g / STAGES) - 1) & 1)) {
                        fail(PCU_DEVERR_EMPTY_WAIT);
                        break;
                    }
                    if (aborted()) break;
                    const uint32_t kdst = base_u32 + SMEM_KV + (2 * s) * TILE_BYTES;
                    const uint32_t vdst = kdst + TILE_BYTES;
                    mbar_arrive_expect_tx(&bars[B_KV_FULL + s], 2 * TILE_BYTES);
                    tma_load_3d(kdst, &tm_k, 0, j * BN, zk, &bars[B_KV_FULL + s]);
                    tma_load_3d(kdst + HALF_BYTES, &tm_k, 64, j * BN, zk, &bars[B_KV_FULL + s]);
                    tma_load_3d(vdst, &tm_v, 0, j * BN, zk, &bars[B_KV_FULL + s]);
                    tma_load_3d(vdst + HALF_BYTES, &tm_v, 64, j * BN, zk, &bars[B_KV_FULL + s]);
                    s_kv_issued = g + 1;
                }
                if (aborted()) break;
            }
        }
    } else if (warp == WARP_MMA) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t qA = base_u32 + SMEM_Q, qB = qA + TILE_BYTES;
            const uint32_t sA = tmem, sB = tmem + 128, oA = tmem + 256, oB = tmem + 384;
            auto k_addr = [&](int g) { return base_u32 + SMEM_KV + (2 * (g % STAGES)) * TILE_BYTES; };
            bool ok = true;
            int g0 = 0, kv_ready = -1, pa = 0, pb = 0;
            auto wait_kv = [&](int g) {
                if (ok && g > kv_ready) {
                    ok = mbar_wait(&bars[B_KV_FULL + g % STAGES], (g / STAGES) & 1);
                    kv_ready = g;
                }
                tc_fence_after();
            };
            for (int k = 0; ok; ++k) {
                const int slot = k & 1;
                ok = mbar_wait(&bars[B_ITEM_FULL + slot], (k >> 1) & 1);
                if (!ok) break;
                const int idx = *(volatile int*)&s_item[slot];
                mbar_arrive(&bars[B_ITEM_EMPTY + slot]);
                if (idx < 0) break;
                const PrefillItem it = prefill_item(idx, a);
                ok = mbar_wait(&bars[B_Q_FULL], k & 1);
                wait_kv(g0);
                if (!ok) break;
                issue_qk(sA, qA, k_addr(g0));
                mma_commit(&bars[B_S_FULL + 0]);
                issue_qk(sB, qB, k_addr(g0));
                mma_commit(&bars[B_S_FULL + 1]);
                if (it.n_kv_B == 1) mma_commit(&bars[B_Q_FREE]);
                for (int j = 0; ok && j < it.n_kv_B; ++j) {
                    const int g = g0 + j;
                    const uint32_t vaddr = k_addr(g) + TILE_BYTES;
                    if (j < it.n_kv_A) {
                        ok = mbar_wait(&bars[B_P_FULL + 0], pa & 1);
                        ++pa;
                        // O_A is overwritten by the first PV: the previous item's O_A must be read out.
                        if (ok && j == 0 && k > 0) ok = mbar_wait(&bars[B_O_FREE + 0], (k - 1) & 1);
                        if (!ok) break;
                        tc_fence_after();
                        issue_pv(oA, sA, vaddr, j == 0, 0, BN / 32);
                        ok = mbar_wait(&bars[B_P_HI + 0], (pa - 1) & 1);     // same phase as P_FULL_A
                        if (!ok) break;
                        tc_fence_after();
                        issue_pv(oA, sA, vaddr, j == 0, BN / 32, BN / 16);
                        if (j + 1 == it.n_kv_A) mma_commit(&bars[B_O_DONE + 0]);
                        if (j + 1 < it.n_kv_A) {
                            wait_kv(g + 1);
                            if (!ok) break;
                            issue_qk(sA, qA, k_addr(g + 1));
                            mma_commit(&bars[B_S_FULL + 0]);
                        }
                    }
                    ok = mbar_wait(&bars[B_P_FULL + 1], pb & 1);
                    ++pb;
                    if (ok && j == 0 && k > 0) ok = mbar_wait(&bars[B_O_FREE + 1], (k - 1) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    issue_pv(oB, sB, vaddr, j == 0, 0, BN / 32);
                    ok = mbar_wait(&bars[B_P_HI + 1], (pb - 1) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    issue_pv(oB, sB, vaddr, j == 0, BN / 32, BN / 16);
                    if (j + 1 == it.n_kv_B) mma_commit(&bars[B_O_DONE + 1]);
                    if (j + 1 < it.n_kv_B) {
                        wait_kv(g + 1);
                        if (!ok) break;
                        issue_qk(sB, qB, k_addr(g + 1));
                        mma_commit(&bars[B_S_FULL + 1]);
                        // S_B of the item's last K/V tile is its last read of Q_A / Q_B.
                        if (j + 2 == it.n_kv_B) mma_commit(&bars[B_Q_FREE]);
                    }
                    mma_commit(&bars[B_KV_EMPTY + g % STAGES]);
                }
                g0 += it.n_kv_B;
            }
            if (!ok) fail(PCU_DEVERR_MMA_WAIT);
            // Let every MMA this thread issued finish before TMEM can be freed.
            mma_commit(&bars[B_DRAIN]);
            if (!mbar_wait(&bars[B_DRAIN], 0)) record_error(a.err, PCU_DEVERR_DRAIN_WAIT);
        }
    } else {
        // ---------------- softmax: one thread per query row of tile X ----------------
        const int x = warp >> 2;                                  // 0 = tile A, 1 = tile B
        const int row = (warp & 3) * 32 + lane;                   // TMEM lane = row in tile
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_tm = tmem + x * 128 + lane_off, o_tm = tmem + 256 + x * 128 + lane_off;
        int sc = 0;                                               // S_FULL_X phases consumed
        bool ok = true;
        for (int k = 0; ok; ++k) {
            const int slot = k & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_ITEM_FULL + slot], (k >> 1) & 1));
            if (!ok) break;
            const int idx = *(volatile int*)&s_item[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_ITEM_EMPTY + slot]);
            if (idx < 0) break;
            const PrefillItem it = prefill_item(idx, a);
            const int qx0 = it.q0 + x * BM;
            const int q = qx0 + row;
            const int n_kv = x ? it.n_kv_B : it.n_kv_A;
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < n_kv; ++j, ++sc) {
                ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_S_FULL + x], sc & 1));
                if (!ok) break;
                tc_fence_after();
                float s[BN];
                tmem_ld128(s_tm, s);
                const int k0 = j * BN;
                if (k0 + BN - 1 > qx0 || k0 + BN > a.T) {
                    #pragma unroll
                    for (int c = 0; c < BN; ++c)
                        if (k0 + c > q || k0 + c >= a.T) s[c] = -INFINITY;
                }
                // Row maximum with three-input max (sm_100): 63 instructions
                // for 128 columns, four independent chains.
                float mx[4];
                #pragma unroll
                for (int i = 0; i < 4; ++i) mx[i] = s[i];
                #pragma unroll
                for (int c = 4; c < BN - 4; c += 8) {
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) mx[i] = fmax3(mx[i], s[c + 2 * i], s[c + 2 * i + 1]);
                }
                const float m_all = fmax3(fmax3(mx[0], s[BN - 4], s[BN - 3]), fmax3(mx[1], s[BN - 2], s[BN - 1]),
                                          fmaxf(mx[2], mx[3]));
                const float m_tile = m_all * a.scale_log2;
                float alpha = 1.0f;
                const bool grow = m_tile > m_run + RESCALE_THRESHOLD || m_run == -INFINITY;
                if (grow) {
                    alpha = fast_exp2(m_run - m_tile);
                    m_run = m_tile;
                }
                // Column pairs: x * scale - m and the row-sum additions as f32x2
                // (one instruction per pair instead of two). P goes out in two
                // halves (keys 0-63, then 64-127), each followed by an arrival,
                // so the first half of P V runs while the second half is made.
                float2 sm2[4];
                #pragma unroll
                for (int i = 0; i < 4; ++i) sm2[i] = make_float2(0.f, 0.f);
                const float2 sc2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-m_run, -m_run);
                {
                    float pk[BN / 4];
                    #pragma unroll
                    for (int c = 0; c < BN / 2; c += 2) {
                        const float2 xx = ffma2(make_float2(s[c], s[c + 1]), sc2, nm2);
                        const float2 p = make_float2(fast_exp2(xx.x), fast_exp2(xx.y));
                        sm2[(c >> 1) & 3] = fadd2(sm2[(c >> 1) & 3], p);
                        pk[c >> 1] = __uint_as_float(pack_bf16x2(p.x, p.y));
                    }
                    tmem_st32(s_tm, pk);                          // P_X keys [0, 64) over S_X columns [0, 32)
                }
                // O_X rescale before the first half's arrival: S_FULL_X(j)
                // implies PV_X(j-1) finished, and PV_X(j) waits for it.
                if (j > 0 && __any_sync(0xffffffffu, grow)) {
                    #pragma unroll
                    for (int c = 0; c < HD / 32; ++c) {
                        float o[32];
                        tmem_ld32(o_tm + c * 32, o);
                        #pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(o_tm + c * 32, o);
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[B_P_FULL + x]);
                {
                    float pk[BN / 4];
                    #pragma unroll
                    for (int c = BN / 2; c < BN; c += 2) {
                        const float2 xx = ffma2(make_float2(s[c], s[c + 1]), sc2, nm2);
                        const float2 p = make_float2(fast_exp2(xx.x), fast_exp2(xx.y));
                        sm2[(c >> 1) & 3] = fadd2(sm2[(c >> 1) & 3], p);
                        pk[(c - BN / 2) >> 1] = __uint_as_float(pack_bf16x2(p.x, p.y));
                    }
                    tmem_st32(s_tm + BN / 4, pk);                 // keys [64, 128) over columns [32, 64)
                }
                const float2 t = fadd2(fadd2(sm2[0], sm2[1]), fadd2(sm2[2], sm2[3]));
                l_run = l_run * alpha + (t.x + t.y);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[B_P_HI + x]);
            }
            if (!ok) break;
            // Item epilogue: read the O row out of TMEM and release O_X for
            // the next item's first PV.
            ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_O_DONE + x], k & 1));
            if (!ok) break;
            tc_fence_after();
            float o[HD];
            #pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                float oc[32];
                tmem_ld32(o_tm + c * 32, oc);
                #pragma unroll
                for (int i = 0; i < 32; ++i) o[c * 32 + i] = oc[i];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_O_FREE + x]);
            // The warp's 32 rows go out 32 columns at a time through its 4 KB
            // stage, laid out as the 128-byte swizzle of a 32 x 32 F32 box
            // (16-byte chunk i of row r at i ^ (r & 7), no bank conflicts),
            // then one TMA store per chunk. The stores drain asynchronously:
            // the warp waits only before it rewrites the stage, so the last
            // chunk's drain overlaps the next item. Rows >= T lie outside the
            // tensor map and are not written.
            const float inv = 1.0f / (l_run == 0.0f ? 1.0f : l_run);
            unsigned char* stage = base + SMEM_OUT + warp * OUT_STAGE_BYTES;
            const uint32_t stage_u32 = base_u32 + SMEM_OUT + warp * OUT_STAGE_BYTES;
            const int row_base = qx0 + (warp & 3) * 32;
            #pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                if (lane == 0) bulk_wait_read_all();
                __syncwarp();
                #pragma unroll
                for (int i = 0; i < 8; ++i)
                    *reinterpret_cast<float4*>(stage + lane * 128 + ((i ^ (lane & 7)) << 4)) =
                        make_float4(o[c * 32 + 4 * i] * inv, o[c * 32 + 4 * i + 1] * inv,
                                    o[c * 32 + 4 * i + 2] * inv, o[c * 32 + 4 * i + 3] * inv);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_4d(stage_u32, &tm_o, c * 32, it.h, row_base, it.seq);
                    bulk_commit();
                }
            }
        }
        // Stores still in flight must finish before the CTA (and its shared
        // memory) goes away.
        if (lane == 0) bulk_wait_all();
        if (!ok && lane == 0) fail(PCU_DEVERR_FULL_WAIT);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == WARP_TMA && lane == 0 && s_abort) {
        // Copies issued but never consumed must land before shared memory goes
        // away: the last STAGES K/V tiles and the last Q cover every copy that
        // can still be in flight.
        const int issued = s_kv_issued;
        for (int g = issued > STAGES ? issued - STAGES : 0; g < issued; ++g)
            if (!mbar_wait(&bars[B_KV_FULL + g % STAGES], (g / STAGES) & 1)) record_error(a.err, PCU_DEVERR_DRAIN_WAIT);
        if (s_q_issued > 0 && !mbar_wait(&bars[B_Q_FULL], (s_q_issued - 1) & 1))
            record_error(a.err, PCU_DEVERR_DRAIN_WAIT);
    }
    if (warp == WARP_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace tc

inline bool prefill_tc_supported(int D, int G) { return D == tc::HD && G >= 1 && G <= 8; }

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder(char* msg, size_t msg_len) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn) {
            snprintf(msg, msg_len, "cuTensorMapEncodeTiled not available");
            return nullptr;
        }
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return encode;
}

// 3-D tensor map over a head-major BF16 tensor [n_heads][T][D]: box 64 x 128 x 1.
inline int make_tmap(CUtensorMap* map, const void* ptr, int T, int n_heads, char* msg, size_t msg_len) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tmap_encoder(msg, msg_len);
    if (!encode) return -9;
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

// 4-D tensor map over the F32 output ao [n_seqs][T][H][D] (dims D, H, T,
// n_seqs): box 32 x 1 x 32 x 1, i.e. 32 columns of one head for 32 rows,
// with the 128-byte swizzle of the epilogue's stage. The T bound keeps the
// rows past a sequence's end from being written.
inline int make_out_tmap(CUtensorMap* map, float* ao, int n_seqs, int T, int H, char* msg, size_t msg_len) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tmap_encoder(msg, msg_len);
    if (!encode) return -9;
    const cuuint64_t dims[4] = {(cuuint64_t)tc::HD, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)n_seqs};
    const cuuint64_t strides[3] = {(cuuint64_t)tc::HD * 4, (cuuint64_t)H * tc::HD * 4, (cuuint64_t)T * H * tc::HD * 4};
    const cuuint32_t box[4] = {32, 1, 32, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ao, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(msg, msg_len, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
        return -9;
    }
    return 0;
}

// The next-item counter of launches made without a handle (one per device;
// such launches on one device must not overlap).
static __device__ unsigned g_prefill_next_item;

// q: [n_seqs][H][T][D], k/v: [n_seqs][HK][T][D] BF16 (rotated); ao: [n_seqs][T][H][D] F32.
// next_item: a zeroed device counter owned by the caller (null: the shared
// per-device counter above). One persistent CTA per SM.
inline int prefill_tc_launch(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, float* ao,
                             int n_seqs, int T, int H, int HK, int D, float scale, int* err, unsigned* next_item,
                             cudaStream_t st, char* msg, size_t msg_len) {
    if (D != tc::HD) {
        snprintf(msg, msg_len, "tensor-core prefill needs head_dim %d", tc::HD);
        return -6;
    }
    if (reinterpret_cast<uintptr_t>(ao) % 16 != 0) {
        snprintf(msg, msg_len, "output must be 16-byte aligned");
        return -6;
    }
    alignas(64) CUtensorMap tq, tk, tv, to;
    if (make_tmap(&tq, q, T, n_seqs * H, msg, msg_len) || make_tmap(&tk, k, T, n_seqs * HK, msg, msg_len) ||
        make_tmap(&tv, v, T, n_seqs * HK, msg, msg_len) || make_out_tmap(&to, ao, n_seqs, T, H, msg, msg_len))
        return -9;
    int device = 0, sms = 0;
    if (cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
        snprintf(msg, msg_len, "device query failed");
        return -9;
    }
    if (!next_item) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_prefill_next_item) != cudaSuccess) {
            snprintf(msg, msg_len, "cudaGetSymbolAddress failed");
            return -9;
        }
        next_item = static_cast<unsigned*>(ptr);
    }
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
    a.n_qb = (T + 2 * tc::BM - 1) / (2 * tc::BM);
    a.n_seqs = n_seqs;
    a.n_items = n_seqs * a.n_qb * H;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.next_item = next_item;
    a.err = err;
    const int grid = a.n_items < sms ? a.n_items : sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(tc::THREADS);
    cfg.dynamicSmemBytes = tc::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, tc::prefill_tc_kernel, tq, tk, tv, to, a);
    if (e != cudaSuccess) {
        snprintf(msg, msg_len, "prefill_tc launch: %s", cudaGetErrorString(e));
        return -9;
    }
    return 0;
}
