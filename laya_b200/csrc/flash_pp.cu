// flash_pp.cu — the attention forward on the 5th-generation tensor cores, two query tiles per CTA in ping-pong
// (head_dim 64).
//
// Contract (Ops.AttentionForward/ForwardUnit, Laya.Training/Ops.cs:260-366): per (segment, head), q and k already
// rotated by the prep pass, sliding layers see keys [i - W, i + W], dropout on the probabilities by the reference's
// counter hash, row log-sum-exp kept for the backward.
//
// One CTA (one per SM, persistent) walks work items (256-query pair tile, head).  The pair's two 128-query tiles A
// and B share one stream of 128-key K/V tiles (a sliding layer's A uses the stream's first tiles, B its last), and
// run as two independent chains on the tensor core, so one tile's softmax overlaps the other's MMAs:
//   warp 0      TMA producer: Q of A and B once per item, then K and V tiles through a STAGES-deep ring.
//   warp 1      TMEM owner and MMA issuer (one thread): S_X = Q_X·Kᵀ into TMEM columns [128·X, 128·X + 128)
//               (M 128, N 128, K 64), O_X += P_X·V into [256 + 128·slot + 64·X, +64) — two O slots alternating by
//               item, so an item's first P·V need not wait for the previous item's epilogue — with P_X read from TMEM (the A operand
//               of the P·V MMA), in the order … P·V_A(j), S_A(j + 1), P·V_B(j), S_B(j + 1) ….  P_X(j) lives in the
//               columns of S_X(j); S_X(j + 1) is issued after P·V_X(j), and MMAs issued by one thread run in order.
//   warps 2-5   softmax of tile A, warps 6-9 of tile B: one thread per query row holds the row's 128 scores, so the
//               row max needs no exchange; it rescales O_X in TMEM when the running max moves (rarely: lazy
//               rescaling), writes P_X in bf16 (hi and lo parts in the accurate forward) over S_X, and at the end
//               stores the context row and its log-sum-exp.
// The commit that signals S_X(j + 1) also covers P·V_X(j) (a commit tracks every earlier MMA of the thread), so a
// softmax thread that sees S_X(j + 1) may rescale O_X and overwrite P_X(j).
// The accurate forward (SPLIT) keeps hi and lo bf16 parts of Q, K, V and P and issues three MMAs per product
// (hi·hi + lo·hi + hi·lo) into the same accumulator.  INFER 1/2: the decision forward's fp16 operands with the
// context as Q8_0 codes (1) or bf16 hi/lo parts (2).
// Every wait is bounded (common.cuh): a protocol fault ends with an error status, never a hung GPU.
#include "common.cuh"
#include "internal.h"
#include "train.h"

namespace laya {
namespace fpp {

constexpr int BQ = 128, BK = 128, HD = 64;
constexpr int TILE = 128 * 128;   // bytes of one 128-row × 64-column 16-bit tile
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_GAP = 8.0f;   // e^8: the largest probability before the running max is raised

template <bool SPLIT>
struct Cfg {
    static constexpr int NQ = SPLIT ? 2 : 1;          // parts of a Q tile (hi, lo)
    static constexpr int NKV = SPLIT ? 4 : 2;         // tiles per ring stage: K, V (+ K lo, V lo)
    static constexpr int STAGES = SPLIT ? 2 : 3;
    static constexpr int TILES = 2 * NQ + STAGES * NKV;
    static constexpr int SMEM = 1024 + TILES * TILE + 256;
    static_assert(SMEM <= 232448, "shared memory budget");
};

struct Params {
    const int32_t* seg_start; const int32_t* seg_len;
    const int32_t* tp_item; const int32_t* tp_p0; const int32_t* n_tp;   // 256-query pair tiles
    int window, hidden, heads;
    float scale, dropout, keep;
    uint64_t seed;
    __nv_bfloat16* out; __nv_bfloat16* out_lo; int ldo;
    float* lse;
    int* err;
    __half* q8; float* q8d; int q8ldd;   // INFER 1: the context as Q8_0 codes [T, hidden] and scales [hidden/32, ldd]
    const uint32_t* dmask; int dmask_w, dmask_rows;   // DROP 2: precomputed dropout decisions (fa::Args)
};

// MN-major operand, 128-byte swizzle (V as the N-contiguous B of P·V): 64-element atoms, 8-row K groups 1024 B apart.
DEVI uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// D[tmem] (+)= A[tmem] · B[smem]: A (M 128 rows in the TMEM lanes, K 16 packed two 16-bit values per column) read
// from tensor memory.
DEVI void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

DEVI void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
DEVI void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
DEVI void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

DEVI uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
DEVI uint32_t pack2h(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
// the bf16 remainders of a pair already packed as `hi`: (a − hi.x, b − hi.y) in bf16
DEVI uint32_t pack2_lo(float a, float b, uint32_t hi) {
    return pack2(__fsub_rn(a, __uint_as_float(hi << 16)), __fsub_rn(b, __uint_as_float(hi & 0xFFFF0000u)));
}
DEVI float lo_part(float x) { return x - __bfloat162float(__float2bfloat16_rn(x)); }
// 2^x by the special-function unit (ex2.approx: ~2 ulp; 2^-inf = 0)
DEVI float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Ops.Uniform (Ops.cs:227-234) at (head << 42) | (row << 21) | key walked along consecutive keys of one row: the first
// step's z = seed + (idx + 1)·φ advances by φ per key, and only bits 40..63 of the final value are used — those
// equal bits 40..63 of the last product (the final xor-shift by 31 cannot reach them), so the last multiply keeps
// only its high word.  u < dropout is compared as the integer bits < ceil(dropout · 2^24): the same test.
struct DropWalk {
    uint64_t z, step;
    uint32_t thr;
    float keep;
    DEVI DropWalk(uint64_t seed, int head, int row, int key, float dropout, float keep_) {
        const uint64_t idx = (static_cast<uint64_t>(head) << 42) | (static_cast<uint64_t>(row) << 21) | static_cast<uint32_t>(key);
        z = seed + (idx + 1ull) * 0x9E3779B97F4A7C15ull;
        step = 0x9E3779B97F4A7C15ull;
        thr = static_cast<uint32_t>(ceilf(dropout * 16777216.0f));
        keep = keep_;
    }
    DEVI float next() {
        uint64_t x = z ^ (z >> 30);
        z += step;
        x *= 0xBF58476D1CE4E5B9ull;
        x ^= x >> 27;
        const uint32_t lo = static_cast<uint32_t>(x), hi = static_cast<uint32_t>(x >> 32);
        const uint32_t c_lo = 0x133111EBu, c_hi = 0x94D049BBu;   // 0x94D049BB133111EB
        const uint32_t top = __umulhi(lo, c_lo) + lo * c_hi + hi * c_lo;
        return (top >> 8) < thr ? 0.0f : keep;
    }
};

// The geometry of one work item: the pair tile's rows, the key stream shared by its two query tiles, and for each
// tile X the range [jlo, jhi) of stream tiles it sees (empty when the tile lies past the segment's end).
struct Span {
    int head, seg0, L, p0, kb, nk;
    int jlo[2], jhi[2];
};
DEVI Span span_of(const Params& p, int item) {
    Span s;
    const int tile = item / p.heads;
    s.head = item - tile * p.heads;
    const int it = p.tp_item[tile];
    s.p0 = p.tp_p0[tile];
    s.seg0 = p.seg_start[it];
    s.L = p.seg_len[it];
    const bool global = p.window < 0;
    const int W = p.window;
    const int rend = min(s.L, s.p0 + 2 * BQ);   // one past the pair's last row
    s.kb = global ? 0 : max(0, s.p0 - W);
    const int ke = global ? s.L : min(s.L, rend + W);
    s.nk = (ke - s.kb + BK - 1) / BK;
#pragma unroll
    for (int x = 0; x < 2; ++x) {
        const int r0 = s.p0 + x * BQ;
        if (r0 >= s.L) { s.jlo[x] = s.jhi[x] = 0; continue; }
        const int r1 = min(s.L, r0 + BQ);
        const int klo = global ? 0 : max(0, r0 - W);
        const int khi = global ? s.L : min(s.L, r1 + W);
        s.jlo[x] = (klo - s.kb) / BK;
        s.jhi[x] = (khi - s.kb + BK - 1) / BK;
    }
    return s;
}

// DROP: 0 no dropout, 1 the counter hash per probability, 2 the precomputed decisions (Params::dmask; global window).
template <bool SPLIT, int DROP, int INFER = 0>
__global__ void __launch_bounds__(320, 1)
    fwd_pp_kernel(const __grid_constant__ CUtensorMap tmh, const __grid_constant__ CUtensorMap tml, Params p) {
    static_assert(!INFER || (!SPLIT && !DROP), "the inference form is single-pass without dropout");
    constexpr bool Q8OUT = INFER == 1, HILO = SPLIT || INFER == 2;
    using C = Cfg<SPLIT>;
    constexpr int S = C::STAGES;
    constexpr uint32_t OPF = INFER ? 0u : 1u;                                       // f16 : bf16
    constexpr uint32_t IDESC_S = make_idesc(1, OPF, OPF, BQ, BK);                   // K-major A, B
    constexpr uint32_t IDESC_PV = make_idesc(1, OPF, OPF, BQ, HD) | (1u << 16);     // A from TMEM; B (V) MN-major
    const int n_items = *p.n_tp * p.heads;
    if (static_cast<int>(blockIdx.x) >= n_items) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                                   // [2 tiles][NQ parts]
    uint8_t* sKV = smem + 2 * C::NQ * TILE;               // [STAGES][NKV]: K, V, K lo, V lo
    uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + S * C::NKV * TILE);
    uint64_t* q_full = bars;
    uint64_t* q_empty = bars + 1;
    uint64_t* s_full = bars + 2;        // [2] by tile
    uint64_t* p_full = bars + 4;        // [2]
    uint64_t* o_done = bars + 6;        // [2]
    uint64_t* o_free = bars + 8;        // [2 tiles][2 O slots]
    uint64_t* kv_full = bars + 12;      // [S]
    uint64_t* kv_empty = bars + 12 + S; // [S]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12 + 2 * S);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = warp_id(), lane = lane_id();
    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int x = 0; x < 2; ++x) {
            mbar_init(s_full + x, 1);
            mbar_init(p_full + x, 4);
            mbar_init(o_done + x, 1);
            mbar_init(o_free + 2 * x, 4);
            mbar_init(o_free + 2 * x + 1, 4);
        }
        for (int s = 0; s < S; ++s) { mbar_init(kv_full + s, 1); mbar_init(kv_empty + s, 1); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmh); if (SPLIT) prefetch_tmap(&tml); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0, n = 0;   // stream tiles and items loaded so far
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
                const Span sp = span_of(p, item);
                const int xq = sp.head * HD, xk = p.hidden + sp.head * HD, xv = 2 * p.hidden + sp.head * HD;
                if (!mbar_wait(q_empty, (n & 1) ^ 1, abort_flag, p.err)) break;
                mbar_arrive_expect_tx(q_full, 2 * C::NQ * TILE);
#pragma unroll
                for (int x = 0; x < 2; ++x) {
                    tma_load_2d(sQ + x * C::NQ * TILE, &tmh, q_full, xq, sp.seg0 + sp.p0 + x * BQ);
                    if constexpr (SPLIT) tma_load_2d(sQ + x * C::NQ * TILE + TILE, &tml, q_full, xq, sp.seg0 + sp.p0 + x * BQ);
                }
                // warm L2 for what comes after the ring's reach: this item's tiles two ahead, the next item's Q and
                // first K/V tiles (the ring cannot hold them yet, so their first loads would otherwise wait on DRAM)
                auto warm = [&](int j) {
                    const int y = sp.seg0 + sp.kb + j * BK;
                    tma_prefetch_2d(&tmh, xk, y);
                    tma_prefetch_2d(&tmh, xv, y);
                    if constexpr (SPLIT) { tma_prefetch_2d(&tml, xk, y); tma_prefetch_2d(&tml, xv, y); }
                };
                if (item + static_cast<int>(gridDim.x) < n_items) {
                    const Span nx = span_of(p, item + gridDim.x);
                    const int nq = nx.head * HD, nk_ = p.hidden + nx.head * HD, nv = 2 * p.hidden + nx.head * HD;
#pragma unroll
                    for (int x = 0; x < 2; ++x) {
                        tma_prefetch_2d(&tmh, nq, nx.seg0 + nx.p0 + x * BQ);
                        if constexpr (SPLIT) tma_prefetch_2d(&tml, nq, nx.seg0 + nx.p0 + x * BQ);
                    }
                    for (int j = 0; j < min(2, nx.nk); ++j) {
                        const int y = nx.seg0 + nx.kb + j * BK;
                        tma_prefetch_2d(&tmh, nk_, y);
                        tma_prefetch_2d(&tmh, nv, y);
                        if constexpr (SPLIT) { tma_prefetch_2d(&tml, nk_, y); tma_prefetch_2d(&tml, nv, y); }
                    }
                }
                for (int j = 0; j < sp.nk; ++j, ++g) {
                    const int s = g % S;
                    if (j + S < sp.nk) warm(j + S);
                    if (!mbar_wait(kv_empty + s, ((g / S) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    uint8_t* st = sKV + s * C::NKV * TILE;
                    const int y = sp.seg0 + sp.kb + j * BK;
                    mbar_arrive_expect_tx(kv_full + s, C::NKV * TILE);
                    tma_load_2d(st, &tmh, kv_full + s, xk, y);
                    tma_load_2d(st + TILE, &tmh, kv_full + s, xv, y);
                    if constexpr (SPLIT) {
                        tma_load_2d(st + 2 * TILE, &tml, kv_full + s, xk, y);
                        tma_load_2d(st + 3 * TILE, &tml, kv_full + s, xv, y);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t base = 0, n = 0, pc[2] = {0, 0}, oc[2] = {0, 0};
            bool ok = true;
            Span nx = span_of(p, blockIdx.x);
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
                const Span sp = nx;
                // the next item's geometry is read now, so its latency overlaps this item's MMAs
                if (item + static_cast<int>(gridDim.x) < n_items) nx = span_of(p, item + gridDim.x);
                if (!mbar_wait(q_full, n & 1, abort_flag, p.err)) break;
                tc_fence_after();
                int s_left = (sp.jhi[0] - sp.jlo[0]) + (sp.jhi[1] - sp.jlo[1]);
                int next_s[2] = {sp.jlo[0], sp.jlo[1]};   // the next stream tile whose scores tile X needs
                // S_X(j) = Q_X · K_jᵀ
                auto issue_s = [&](int x, int j) -> bool {
                    const uint32_t g = base + j;
                    const int s = g % S;
                    if (!mbar_wait(kv_full + s, (g / S) & 1, abort_flag, p.err)) return false;
                    tc_fence_after();
                    const uint32_t ak = smem_u32(sKV + s * C::NKV * TILE), akl = ak + 2 * TILE;
                    const uint32_t aq = smem_u32(sQ + x * C::NQ * TILE), aql = aq + TILE;
                    const uint32_t d = tmem + x * BK;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        mma_f16(d, smem_desc_sw128(aq + kk * 32), smem_desc_sw128(ak + kk * 32), IDESC_S, kk > 0);
                    if constexpr (SPLIT) {
#pragma unroll
                        for (int kk = 0; kk < HD / 16; ++kk) {
                            mma_f16(d, smem_desc_sw128(aql + kk * 32), smem_desc_sw128(ak + kk * 32), IDESC_S, 1u);
                            mma_f16(d, smem_desc_sw128(aq + kk * 32), smem_desc_sw128(akl + kk * 32), IDESC_S, 1u);
                        }
                    }
                    mma_commit(s_full + x);
                    next_s[x] = j + 1;
                    if (--s_left == 0) mma_commit(q_empty);   // Q free once the item's last scores are done
                    return true;
                };
                // O_X (+)= P_X(j) · V_j, P_X in the TMEM columns of S_X
                auto issue_pv = [&](int x, int j) -> bool {
                    const bool first = j == sp.jlo[x];
                    if (!mbar_wait(p_full + x, pc[x]++ & 1, abort_flag, p.err)) return false;
                    // O_X alternates between two TMEM slots by item; the item's first P·V overwrites its slot, which
                    // the epilogue of the item two back must have read
                    const uint32_t slot = oc[x] & 1;
                    if (first && !mbar_wait(o_free + 2 * x + slot, ((oc[x] >> 1) & 1) ^ 1, abort_flag, p.err)) return false;
                    tc_fence_after();
                    const uint32_t g = base + j;
                    const int s = g % S;
                    const uint32_t av = smem_u32(sKV + s * C::NKV * TILE) + TILE, avl = av + 2 * TILE;
                    const uint32_t tp = tmem + x * BK, tpl = tp + BK / 2, to = tmem + 2 * BK + slot * 2 * HD + x * HD;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_ts(to, tp + kk * 8, desc_mn_sw128(av + kk * 2048, TILE), IDESC_PV, (!first || kk > 0) ? 1u : 0u);
                    if constexpr (SPLIT) {
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            mma_ts(to, tpl + kk * 8, desc_mn_sw128(av + kk * 2048, TILE), IDESC_PV, 1u);
                            mma_ts(to, tp + kk * 8, desc_mn_sw128(avl + kk * 2048, TILE), IDESC_PV, 1u);
                        }
                    }
                    if (j == sp.jhi[x] - 1) { mma_commit(o_done + x); ++oc[x]; }
                    return true;
                };
                // both tiles' first scores as soon as their K tiles are in (the ring holds the first two)
                for (int x = 0; x < 2 && ok; ++x)
                    if (sp.jlo[x] < sp.jhi[x] && sp.jlo[x] < S) ok = issue_s(x, sp.jlo[x]);
                for (int j = 0; j < sp.nk && ok; ++j) {
                    if (j >= sp.jlo[0] && j < sp.jhi[0]) {
                        if (!(ok = issue_pv(0, j))) break;
                        if (j + 1 < sp.jhi[0] && next_s[0] == j + 1 && !(ok = issue_s(0, j + 1))) break;
                    }
                    if (j >= sp.jlo[1] && j < sp.jhi[1] && !(ok = issue_pv(1, j))) break;
                    mma_commit(kv_empty + (base + j) % S);   // every MMA reading K_j and V_j is issued
                    for (int x = 0; x < 2 && ok; ++x)
                        if (j + 1 >= sp.jlo[x] && j + 1 < sp.jhi[x] && next_s[x] == j + 1) ok = issue_s(x, j + 1);
                }
                base += sp.nk;
            }
        }
    } else {
        // softmax: tile X = (warp − 2) / 4; thread = one query row of that tile, in the warp's TMEM lane quarter
        const int x = (warp - 2) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t tS = tmem + lane_off + x * BK;
        const bool global = p.window < 0;
        const int W = p.window;
        const float c2 = p.scale * LOG2E;           // scores → log2 units
        const float gap = RESCALE_GAP / p.scale;    // the rescale threshold in raw score units
        uint32_t sc = 0, oc = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            const Span sp = span_of(p, item);
            if (sp.jlo[x] >= sp.jhi[x]) continue;
            const int q = sp.p0 + x * BQ + row;
            // keys this row sees: [lo, lo + span]; a row past the segment sees none (k − lo > 0 = span for every key)
            const bool qin = q < sp.L;
            const int lo = qin ? (global ? 0 : max(0, q - W)) : -(1 << 30);
            const uint32_t span = qin ? static_cast<uint32_t>((global ? sp.L - 1 : min(sp.L - 1, q + W)) - lo) : 0u;
            const uint32_t oslot = oc & 1;   // this item's O slot (the MMA thread alternates them the same way)
            const uint32_t tO = tmem + lane_off + 2 * BK + oslot * 2 * HD + x * HD;
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = sp.jlo[x]; j < sp.jhi[x]; ++j) {
                ok = __all_sync(0xffffffffu, ok && mbar_wait(s_full + x, sc++ & 1, abort_flag, p.err));
                if (!ok) break;
                tc_fence_after();
                const int k0 = sp.kb + j * BK;
                uint32_t v[BK];
#pragma unroll
                for (int c = 0; c < BK / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
                tmem_ld_wait();
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                const bool whole = static_cast<uint32_t>(k0 - lo) <= span && static_cast<uint32_t>(k0 + BK - 1 - lo) <= span;
                if (__all_sync(0xffffffffu, whole)) {
#pragma unroll
                    for (int e = 0; e < BK; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(v[e]));
                } else {
#pragma unroll
                    for (int e = 0; e < BK; ++e) {
                        const bool vis = static_cast<uint32_t>(k0 + e - lo) <= span;
                        const float s = vis ? __uint_as_float(v[e]) : -INFINITY;
                        v[e] = __float_as_uint(s);
                        mx4[e & 3] = fmaxf(mx4[e & 3], s);
                    }
                }
                const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
                // Lazy rescaling: the running max moves only when the tile's max exceeds it by more than the gap, so
                // probabilities stay below e^RESCALE_GAP and O is rescaled in TMEM rarely.  Every P of a row and its
                // sum l use the same reference max.
                const bool grow = mx > m_run + gap;
                const float m_new = grow ? mx : m_run;
                const float alpha = m_run == -INFINITY ? 0.f : (grow ? ex2(__fmul_rn(m_run - m_new, c2)) : 1.0f);
                const float msc = m_new == -INFINITY ? 0.f : m_new * c2;
                // P = 2^(s·c2 − m·c2); the row sum counts every probability, dropped or not.  32 keys at a time into
                // the TMEM columns of S: hi parts at [0, 64), lo parts at [64, 128)
                // (pairs of keys in the two lanes of f32x2 registers: one instruction per pair for the exponent's
                // argument, the row sum and the lo remainder)
                uint64_t rs2[2] = {0ull, 0ull};
                const uint64_t c2x2 = f2_pack(c2, c2), nm2 = f2_pack(-msc, -msc);
                DropWalk walk(p.seed, sp.head, sp.seg0 + q, k0, p.dropout, p.keep);
                // precomputed decisions: the row's four words for the tile's 128 keys (k0 is a multiple of 128)
                uint32_t dw[BK / 32] = {0u, 0u, 0u, 0u};
                if (DROP == 2 && qin) {
                    const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(
                        p.dmask + (static_cast<size_t>(sp.head) * p.dmask_rows + sp.seg0 + q) * p.dmask_w + k0 / 32));
                    dw[0] = w4.x; dw[1] = w4.y; dw[2] = w4.z; dw[3] = w4.w;
                }
#pragma unroll
                for (int c = 0; c < BK / 32; ++c) {
                    uint32_t* f = v + 32 * c;   // the probabilities replace the scores
                    uint32_t ph[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const uint64_t arg = f2_fma(f2_pack(__uint_as_float(f[2 * e]), __uint_as_float(f[2 * e + 1])), c2x2, nm2);
                        float a, b;
                        f2_unpack(arg, a, b);
                        a = ex2(a);   // 2^-inf = 0 when masked
                        b = ex2(b);
                        const uint64_t pr = f2_pack(a, b);
                        rs2[e & 1] = f2_add(rs2[e & 1], pr);
                        if constexpr (DROP == 2) {
                            a = (dw[c] >> (2 * e)) & 1u ? a * p.keep : 0.f;
                            b = (dw[c] >> (2 * e + 1)) & 1u ? b * p.keep : 0.f;
                        } else if constexpr (DROP == 1) {
                            a *= walk.next();
                            b *= walk.next();
                        }
                        ph[e] = INFER ? pack2h(a, b) : pack2(a, b);
                        if constexpr (SPLIT) {   // keep P for the lo remainder
                            f[2 * e] = __float_as_uint(a);
                            f[2 * e + 1] = __float_as_uint(b);
                        }
                    }
                    tmem_st16(tS + c * 16, ph);
                    if constexpr (SPLIT) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const uint64_t hi = f2_pack(__uint_as_float(ph[e] << 16), __uint_as_float(ph[e] & 0xFFFF0000u));
                            float a, b;
                            f2_unpack(f2_sub(f2_pack(__uint_as_float(f[2 * e]), __uint_as_float(f[2 * e + 1])), hi), a, b);
                            ph[e] = pack2(a, b);
                        }
                        tmem_st16(tS + BK / 2 + c * 16, ph);
                    }
                }
                float rs_a, rs_b, rs_c, rs_d;
                f2_unpack(rs2[0], rs_a, rs_b);
                f2_unpack(rs2[1], rs_c, rs_d);
                const float rsum = (rs_a + rs_b) + (rs_c + rs_d);
                // O_X is complete up to tile j − 1 (the commit behind s_full covers that P·V): rescale it in place,
                // 32 columns at a time, before P·V_X(j) adds to it
                if (j > sp.jlo[x] && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                    for (int h = 0; h < HD / 32; ++h) {
                        uint32_t o[32];
                        tmem_ld32(tO + h * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st32(tO + h * 32, o);
                    }
                }
                l_run = l_run * alpha + rsum;
                m_run = m_new;
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full + x);
            }
            // the context row once the item's last P·V of this tile is done
            ok = __all_sync(0xffffffffu, ok && mbar_wait(o_done + x, oc++ & 1, abort_flag, p.err));
            if (!ok) break;
            tc_fence_after();
            uint32_t o[HD];
            tmem_ld32(tO, *reinterpret_cast<uint32_t(*)[32]>(o));
            tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
            tmem_ld_wait();
            // O_X is in registers: the item two ahead may overwrite this slot
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free + 2 * x + oslot);
            if (!qin) continue;
            const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
            const size_t tok = static_cast<size_t>(sp.seg0 + q);
            if constexpr (Q8OUT) {
#pragma unroll
                for (int blk = 0; blk < HD / 32; ++blk) {
                    float f[32];
                    float m = 0.f;
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        f[e] = __uint_as_float(o[32 * blk + e]) * inv;
                        m = fmaxf(m, fabsf(f[e]));
                    }
                    const float id = m != 0.0f ? __fdiv_rn(127.0f, m) : 0.0f;
                    __half* qrow = p.q8 + tok * p.hidden + sp.head * HD + blk * 32;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        __half hq[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) hq[e] = __int2half_rn(__float2int_rn(__fmul_rn(f[8 * t + e], id)));
                        *reinterpret_cast<uint4*>(qrow + 8 * t) = *reinterpret_cast<const uint4*>(hq);
                    }
                    p.q8d[static_cast<size_t>(sp.head * 2 + blk) * p.q8ldd + tok] = round_fp16(__fdiv_rn(m, 127.0f));
                }
            } else {
                __nv_bfloat16* orow = p.out + tok * p.ldo + sp.head * HD;
#pragma unroll
                for (int t = 0; t < HD / 8; ++t) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[8 * t + e]) * inv;
                    *reinterpret_cast<uint4*>(orow + 8 * t) =
                        make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                    if constexpr (HILO) {
                        __nv_bfloat16* lrow = p.out_lo + tok * p.ldo + sp.head * HD;
                        *reinterpret_cast<uint4*>(lrow + 8 * t) =
                            make_uint4(pack2(lo_part(f[0]), lo_part(f[1])), pack2(lo_part(f[2]), lo_part(f[3])),
                                       pack2(lo_part(f[4]), lo_part(f[5])), pack2(lo_part(f[6]), lo_part(f[7])));
                    }
                }
                if (!INFER) p.lse[tok * p.heads + sp.head] = m_run * p.scale + logf(l_run);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace fpp

template <bool SPLIT, int DROP>
static int launch_pp(const fa::Args& a, cudaStream_t s) {
    using C = fpp::Cfg<SPLIT>;
    CUtensorMap th, tl;
    int rc = make_tmap_2d(&th, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                          static_cast<uint64_t>(a.ld) * 2, fpp::BK, fpp::HD, true);
    if (!rc) rc = make_tmap_2d(&tl, SPLIT ? a.qkv_lo : a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                               static_cast<uint64_t>(a.ld) * 2, fpp::BK, fpp::HD, true);
    if (rc) return rc;
    static DeviceOnce attr;
    int dev = 0, nsm = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(fpp::fwd_pp_kernel<SPLIT, DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM));
        attr.mark(dev);
    }
    if (int e = sm_count(dev, &nsm)) return e;
    fpp::Params p{};
    p.seg_start = a.seg_start; p.seg_len = a.seg_len;
    p.tp_item = a.tp_item; p.tp_p0 = a.tp_p0; p.n_tp = a.n_tp;
    p.window = a.window; p.hidden = a.hidden; p.heads = a.heads;
    p.scale = a.scale; p.dropout = a.dropout; p.keep = a.keep; p.seed = a.seed;
    p.out = a.out; p.out_lo = a.out_lo; p.ldo = a.ldo; p.lse = a.lse; p.err = a.err;
    p.dmask = a.dmask; p.dmask_w = a.dmask_w; p.dmask_rows = a.dmask_rows;
    const int items = a.max_tp * a.heads;
    fpp::fwd_pp_kernel<SPLIT, DROP><<<items < nsm ? items : nsm, 320, C::SMEM, s>>>(th, tl, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

// The dropout decisions of one layer (Ops.Dropout's counter hash, walked along keys as the forward walks them): one
// warp per (head, row), each lane 32 keys of the row's segment at a time, one bit per key (1: kept).
__global__ void __launch_bounds__(256) drop_mask_kernel(uint64_t seed, float dropout, float keep, int heads, int T,
                                                        const int32_t* __restrict__ tok_item,
                                                        const int32_t* __restrict__ seg_len, uint32_t* __restrict__ mask,
                                                        int rows, int mw) {
    const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= static_cast<long long>(heads) * T) return;
    const int h = static_cast<int>(wid / T), t = static_cast<int>(wid % T);
    const int nw = min((seg_len[tok_item[t]] + 31) / 32, mw);
    for (int w = lane; w < nw; w += 32) {
        fpp::DropWalk walk(seed, h, t, 32 * w, dropout, keep);
        uint32_t bits = 0;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) bits |= (walk.next() != 0.f ? 1u : 0u) << i;
        mask[(static_cast<size_t>(h) * rows + t) * mw + w] = bits;
    }
}

int drop_mask(const fa::Args& a, const int32_t* tok_item, uint32_t* mask, cudaStream_t s) {
    if (a.T <= 0 || a.dropout <= 0.f) return OK;
    if (!mask || a.dmask_w <= 0 || (a.dmask_w & 3) || a.dmask_rows < a.T || !tok_item) return ERR_ARGUMENT;
    const long long threads = static_cast<long long>(a.heads) * a.T * 32;
    drop_mask_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(
        a.seed, a.dropout, a.keep, a.heads, a.T, tok_item, a.seg_len, mask, a.dmask_rows, a.dmask_w);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

// The training forward on the tensor cores for head_dim 64, two query tiles per CTA; ERR_NOT_SUPPORTED for shapes it
// does not take (the caller then runs another form).
int flash_forward_pp(const fa::Args& a, cudaStream_t s) {
    if (a.hidden / a.heads != fpp::HD || !a.tp_item || a.max_tp <= 0 || a.T <= 0) return ERR_NOT_SUPPORTED;
    if ((a.ld & 7) || (reinterpret_cast<uintptr_t>(a.qkv) & 15) || (a.qkv_lo && (reinterpret_cast<uintptr_t>(a.qkv_lo) & 15)))
        return ERR_NOT_SUPPORTED;
    if (a.qkv_lo && !a.out_lo) { set_error("accurate attention needs the context's low part"); return ERR_ARGUMENT; }
    const int drop = a.dropout <= 0.f ? 0 : (a.dmask && a.window < 0 ? 2 : 1);
    if (a.qkv_lo) return drop == 2 ? launch_pp<true, 2>(a, s) : drop ? launch_pp<true, 1>(a, s) : launch_pp<true, 0>(a, s);
    return drop == 2 ? launch_pp<false, 2>(a, s) : drop ? launch_pp<false, 1>(a, s) : launch_pp<false, 0>(a, s);
}

}  // namespace laya
