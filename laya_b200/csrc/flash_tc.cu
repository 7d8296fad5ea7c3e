// flash_tc.cu — the fine-tune attention forward on the 5th-generation tensor cores (head_dim 64).
//
// Same contract as fa::fwd_kernel (flash.cu; Ops.AttentionForward/ForwardUnit, Laya.Training/Ops.cs:260-366):
// per (segment, head), q and k already rotated by the prep pass, sliding layers see keys [i - W, i + W], dropout on
// the probabilities by the reference's counter hash, row log-sum-exp kept for the backward.  One CTA owns 128
// queries of one head:
//   warp 0      TMA producer: the Q tile once, then 128-key K and V tiles through a 2-stage ring.
//   warp 1      TMEM owner and MMA issuer (one thread): S = Q·Kᵀ into one of two TMEM score buffers (columns
//               [0, 128) and [128, 256); M 128, N 128, K 64), and O += P·V into columns [256, 320) (M 128, N 64,
//               K 128; V read N-contiguous).  The scores of tile j + 1 are issued before P·V of tile j, so they are
//               ready when the softmax warps finish tile j.
//   warps 2-9   softmax: two warps per TMEM lane quarter, so thread (half, i) owns 64 key columns of query row i.
//               Per key tile it reads its half-row of S from TMEM in one round trip, masks it branch-free against the
//               row's visible key range, exchanges the half-row maxima through shared memory (one named barrier),
//               exponentiates and sums, rescales its half of the O row in TMEM when the max moved, and writes its
//               64-key half of P in bf16 into shared memory in the 128-byte-swizzled K-major layout the P·V MMA reads.
//               At the end the two halves' row sums are combined and each warp stores its 32 context columns.
// The accurate forward (SPLIT) keeps hi and lo bf16 parts of Q, K, V and P and issues three MMAs per product
// (hi·hi + lo·hi + hi·lo), accumulating in the same TMEM columns.
// The backward's dK/dV kernel (bwd_dkdv_tc_kernel, below) uses the same roles with keys in the TMEM lanes, and its dQ
// kernel (bwd_dq_tc_kernel) the forward's layout with dP = dO·Vᵀ beside S and dQ += dS·K in place of P·V.
// Every wait is bounded (common.cuh): a protocol fault ends with an error status, never a hung GPU.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "train.h"

namespace laya {
namespace fat {

constexpr int BQ = 128, BK = 128, HD = 64;
constexpr int TILE = 128 * 128;   // bytes of one 128-row × 64-column bf16 tile
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_GAP = 8.0f;   // e^8 ≈ 2981: the largest probability before the running max is raised

template <bool SPLIT>
struct Cfg {
    static constexpr int NQ = SPLIT ? 2 : 1;          // Q tiles (hi, lo)
    static constexpr int NKV = SPLIT ? 4 : 2;         // tiles per ring stage: K, V (+ K lo, V lo)
    static constexpr int STAGES = 2;
    static constexpr int NP = SPLIT ? 2 : 1;          // parts of P (hi, lo), each two 64-key sub-tiles
    static constexpr int NPB = SPLIT ? 1 : 2;         // P buffers: two let the next tile's P be written while P·V runs
    static constexpr int TILES = NQ + STAGES * NKV + 2 * NP * NPB;
    static constexpr int SMEM = 1024 + TILES * TILE + 256 + 2 * BQ * 4;   // + the two halves' row max / row sum
    static_assert(SMEM <= 232448, "shared memory budget");
};

struct Params {
    const int32_t* seg_start; const int32_t* seg_len;
    const int32_t* tq_item; const int32_t* tq_p0; const int32_t* n_tq;
    int window, hidden, heads;
    float scale, dropout, keep;
    uint64_t seed;
    __nv_bfloat16* out; __nv_bfloat16* out_lo; int ldo;
    float* lse;
    int* err;
    __half* q8; float* q8d; int q8ldd;   // inference: the context as Q8_0 codes [T, hidden] and scales [hidden/32, ldd]
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

DEVI uint32_t pack2h(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
DEVI uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
DEVI float lo_part(float x) { return x - __bfloat162float(__float2bfloat16_rn(x)); }
// 2^x by the special-function unit (ex2.approx: ~2 ulp; 2^-inf = 0)
DEVI float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
DEVI void named_bar_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

// Ops.Uniform (Ops.cs:227-234) at (head << 42) | (row << 21) | key, the dropout mask's counter hash.
// The same hash walked along consecutive indices: the first step's z = seed + (idx + 1)·φ advances by a fixed
// multiple of φ per element (one key, or one row = 2^21 indices), and only bits 40..63 of the final value are used —
// those equal bits 40..63 of the last product (the final xor-shift by 31 cannot reach them), so the last multiply
// keeps only its high word.  u < dropout is compared as the integer bits < ceil(dropout · 2^24): the same test.
struct DropWalk {
    uint64_t z, step;
    uint32_t thr;
    float keep;
    DEVI DropWalk(uint64_t seed, int head, int row, int key, uint64_t stride, float dropout, float keep_) {
        const uint64_t idx = (static_cast<uint64_t>(head) << 42) | (static_cast<uint64_t>(row) << 21) | static_cast<uint32_t>(key);
        z = seed + (idx + 1ull) * 0x9E3779B97F4A7C15ull;
        step = stride * 0x9E3779B97F4A7C15ull;
        thr = static_cast<uint32_t>(ceilf(dropout * 16777216.0f));
        keep = keep_;
    }
    // the multiplier of the current index, then advance to the next
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

// Persistent: a CTA walks work items (query tile, head) = blockIdx.x, blockIdx.x + gridDim.x, …, and every barrier
// phase runs on across items (key tiles are counted globally), so the next item's Q and first K/V tiles load and its
// first scores are computed while the softmax warps finish the current item.
// INFER: the decision forward's attention — fp16 Q, K, V and P (kind::f16 with f16 operands), and the context leaves
// as Q8_0 codes for the Wo product: each softmax thread holds one 32-column block of its row (Q8_0.QuantizeActivations,
// PackedMatrixQ8_0.cs:50-71: d = amax/127 stored fp16, q = round-half-even(x · 127/amax)).
// INFER 2: the same fp16 operands with the context as bf16 hi/lo parts (the fp32-accurate decision forward).
template <bool SPLIT, bool DROP, int INFER = 0>
__global__ void __launch_bounds__(320, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmh, const __grid_constant__ CUtensorMap tml, Params p) {
    static_assert(!INFER || (!SPLIT && !DROP), "the inference form is single-pass without dropout");
    constexpr bool Q8OUT = INFER == 1, HILO = SPLIT || INFER == 2;
    using C = Cfg<SPLIT>;
    constexpr uint32_t OPF = INFER ? 0u : 1u;                                                    // f16 : bf16
    constexpr uint32_t IDESC_S = make_idesc(1, OPF, OPF, BQ, BK);                                // K-major A, B
    constexpr uint32_t IDESC_PV = make_idesc(1, OPF, OPF, BQ, HD) | (1u << 16);                  // B (V) MN-major
    const int n_items = *p.n_tq * p.heads;
    if (static_cast<int>(blockIdx.x) >= n_items) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                                   // [NQ] tiles
    uint8_t* sKV = smem + C::NQ * TILE;                   // [STAGES][NKV] tiles: K, V, K lo, V lo
    uint8_t* sP = sKV + C::STAGES * C::NKV * TILE;        // [NPB][NP][2] sub-tiles (keys 0-63, 64-127)
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::NP * C::NPB * TILE);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;       // [2] ring stages
    uint64_t* kv_empty = bars + 3;      // [2]
    uint64_t* s_full = bars + 5;        // [2] S buffers in TMEM
    uint64_t* p_full = bars + 7;        // [2] by tile parity
    uint64_t* o_done = bars + 9;        // [2] by tile parity
    uint64_t* q_empty = bars + 11;      // Q read by the item's last score MMAs
    uint64_t* o_free = bars + 12;       // O read by the item's epilogue
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(bars + 32);   // [2 halves][BQ]: row maxima per tile, then the row sums

    const bool global = p.window < 0;
    const int W = p.window;
    const int warp = warp_id(), lane = lane_id();
    // the key range of an item's query tile
    auto span_of = [&](int item, int& head, int& seg0, int& L, int& q0, int& kb, int& nk) {
        const int tile = item / p.heads;
        head = item - tile * p.heads;
        const int it = p.tq_item[tile];
        q0 = p.tq_p0[tile];
        seg0 = p.seg_start[it];
        L = p.seg_len[it];
        kb = global ? 0 : max(0, q0 - W);
        const int ke = global ? L : min(L, q0 + BQ + W);
        nk = (ke - kb + BK - 1) / BK;
    };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        mbar_init(o_free, 8);
        for (int s = 0; s < 2; ++s) {
            mbar_init(kv_full + s, 1);
            mbar_init(kv_empty + s, 1);
            mbar_init(s_full + s, 1);
            mbar_init(p_full + s, 8);
            mbar_init(o_done + s, 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmh); if (SPLIT) prefetch_tmap(&tml); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tO = tmem + 2 * BK;   // S buffers at columns [0, 128) and [128, 256); O at [256, 320)

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0, n = 0;   // key tiles and items loaded so far
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
                int head, seg0, L, q0, kb, nk;
                span_of(item, head, seg0, L, q0, kb, nk);
                const int xq = head * HD, xk = p.hidden + head * HD, xv = 2 * p.hidden + head * HD;
                if (!mbar_wait(q_empty, (n & 1) ^ 1, abort_flag, p.err)) break;
                mbar_arrive_expect_tx(q_full, C::NQ * TILE);
                tma_load_2d(sQ, &tmh, q_full, xq, seg0 + q0);
                if constexpr (SPLIT) tma_load_2d(sQ + TILE, &tml, q_full, xq, seg0 + q0);
                for (int j = 0; j < nk; ++j, ++g) {
                    const int s = g & 1;
                    if (!mbar_wait(kv_empty + s, ((g >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    uint8_t* st = sKV + s * C::NKV * TILE;
                    const int y = seg0 + kb + j * BK;
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
            // per item, iteration j issues S_j (into TMEM buffer g % 2) and then P·V of tile j − 1, so the scores of
            // the next tile are computed while the softmax warps work on the current one
            uint32_t base = 0, n = 0;
            bool ok = true;
            const uint32_t aq = smem_u32(sQ), aql = smem_u32(sQ + TILE);
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
                int head, seg0, L, q0, kb, nk;
                span_of(item, head, seg0, L, q0, kb, nk);
                if (!mbar_wait(q_full, n & 1, abort_flag, p.err)) break;
                tc_fence_after();
                for (int j = 0; j <= nk; ++j) {
                    if (j < nk) {
                        const uint32_t g = base + j;
                        const int s = g & 1;
                        if (!mbar_wait(kv_full + s, (g >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t ak = smem_u32(sKV + s * C::NKV * TILE), akl = ak + 2 * TILE;
                        const uint32_t d = tS + s * BK;
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
                        mma_commit(s_full + s);
                        if (j == nk - 1) mma_commit(q_empty);   // Q free once the item's last scores are done
                    }
                    if (j >= 1) {
                        const int i = j - 1;
                        const uint32_t gi = base + i;
                        const int s = gi & 1;
                        if (!mbar_wait(p_full + s, (gi >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
                        // the first P·V of an item overwrites O: the previous item's epilogue must have read it
                        if (i == 0 && !mbar_wait(o_free, (n & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t av = smem_u32(sKV + s * C::NKV * TILE) + TILE, avl = av + 2 * TILE;
                        const uint32_t ap = smem_u32(sP + (gi % C::NPB) * C::NP * 2 * TILE), apl = ap + 2 * TILE;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint32_t po = (kk >> 2) * TILE + (kk & 3) * 32;
                            mma_f16(tO, smem_desc_sw128(ap + po), desc_mn_sw128(av + kk * 2048, TILE), IDESC_PV,
                                    (i > 0 || kk > 0) ? 1u : 0u);
                        }
                        if constexpr (SPLIT) {
#pragma unroll
                            for (int kk = 0; kk < BK / 16; ++kk) {
                                const uint32_t po = (kk >> 2) * TILE + (kk & 3) * 32;
                                mma_f16(tO, smem_desc_sw128(apl + po), desc_mn_sw128(av + kk * 2048, TILE), IDESC_PV, 1u);
                                mma_f16(tO, smem_desc_sw128(ap + po), desc_mn_sw128(avl + kk * 2048, TILE), IDESC_PV, 1u);
                            }
                        }
                        mma_commit(o_done + s);
                        mma_commit(kv_empty + s);
                    }
                }
                base += nk;
            }
        }
    } else {
        // softmax: two warps per TMEM lane quarter, each owning 64 of the tile's 128 key columns (and 32 of O's 64)
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        constexpr int HK = BK / 2, HO = HD / 2;
        // `ok` is kept warp-uniform and the loops never exit early: the 256 softmax threads take the same named
        // barriers in every case (an aborted protocol only skips the work between them)
        bool ok = true;
        uint32_t base = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            int head, seg0, L, q0, kb, nk;
            span_of(item, head, seg0, L, q0, kb, nk);
            const int q = q0 + row;
            // keys this row sees: [lo, hi] (empty for rows past the segment)
            const int lo = q < L ? (global ? 0 : max(0, q - W)) : 1;
            const int hi = q < L ? (global ? L - 1 : min(L - 1, q + W)) : 0;
            const uint32_t span = static_cast<uint32_t>(hi - lo);
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < nk; ++j) {
                const uint32_t g = base + j;
                ok = __all_sync(0xffffffffu, ok && mbar_wait(s_full + (g & 1), (g >> 1) & 1, abort_flag, p.err));
                const int k0 = kb + j * BK + half * HK;
                uint32_t v[HK];
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                if (ok) {
                    tc_fence_after();
                    const uint32_t sb = tS + (g & 1) * BK;
#pragma unroll
                    for (int c = 0; c < HK / 32; ++c)
                        tmem_ld32(sb + lane_off + half * HK + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < HK; ++e) {
                        const bool vis = static_cast<uint32_t>(k0 + e - lo) <= span;
                        const float x = vis ? __fmul_rn(__uint_as_float(v[e]), p.scale) : -INFINITY;
                        v[e] = __float_as_uint(x);
                        mx4[e & 3] = fmaxf(mx4[e & 3], x);
                    }
                }
                // the row max over both halves
                red[half * BQ + row] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
                named_bar_sync(1, 256);
                const float mx = fmaxf(red[row], red[BQ + row]);
                named_bar_sync(1, 256);
                if (!ok) continue;
                // Lazy rescaling: the running max moves only when the tile's max exceeds it by more than
                // RESCALE_GAP (natural log units), so probabilities stay below e^RESCALE_GAP and O is rescaled in TMEM
                // rarely.  Every P of a row and its sum l use the same reference max.
                const bool grow = mx > m_run + RESCALE_GAP;
                const float m_new = grow ? mx : m_run;
                const float alpha = (m_run == -INFINITY || !grow) ? (m_run == -INFINITY ? 0.f : 1.0f)
                                                                   : ex2(__fmul_rn(m_run - m_new, LOG2E));
                const float msc = m_new == -INFINITY ? 0.f : m_new * LOG2E;
                // P = exp(s - m); the row sum counts every probability, dropped or not
                float rs4[4] = {0.f, 0.f, 0.f, 0.f};
                DropWalk walk(p.seed, head, seg0 + q, k0, 1, p.dropout, p.keep);
#pragma unroll
                for (int e = 0; e < HK; ++e) {
                    float pe = ex2(fmaf(__uint_as_float(v[e]), LOG2E, -msc));   // 2^-inf = 0 for masked keys
                    rs4[e & 3] += pe;
                    if constexpr (DROP) pe = pe * walk.next();
                    v[e] = __float_as_uint(pe);
                }
                // O may be rescaled only once P·V of the previous tile is done; the P buffer of this tile may be
                // rewritten once the P·V that last read it (tile g − NPB) is done — for an item's first tile the
                // previous item's epilogue already waited for every earlier P·V.  Waiting here, after the
                // exponentials, lets them overlap that P·V.
                const bool rescale = j > 0 && __any_sync(0xffffffffu, alpha != 1.0f);
                if (rescale || j >= C::NPB) {
                    const uint32_t i = rescale ? g - 1 : g - C::NPB;
                    ok = __all_sync(0xffffffffu, mbar_wait(o_done + (i & 1), (i >> 1) & 1, abort_flag, p.err));
                    if (!ok) continue;
                    tc_fence_after();
                    if (rescale) {
                        uint32_t o[HO];
                        tmem_ld32(tO + lane_off + half * HO, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < HO; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st32(tO + lane_off + half * HO, o);
                        tmem_st_wait();
                    }
                }
                // this half's 64 keys are sub-tile `half` of P buffer g % NPB: 16-byte chunk c of row `row`,
                // swizzled by row % 8
                uint8_t* prow = sP + (g % C::NPB) * C::NP * 2 * TILE + half * TILE + row * 128;
#pragma unroll
                for (int c = 0; c < HK / 8; ++c) {
                    const float* f = reinterpret_cast<const float*>(v + 8 * c);
                    uint8_t* dst = prow + ((c ^ (row & 7)) << 4);
                    if constexpr (INFER)
                        *reinterpret_cast<uint4*>(dst) = make_uint4(pack2h(f[0], f[1]), pack2h(f[2], f[3]),
                                                                    pack2h(f[4], f[5]), pack2h(f[6], f[7]));
                    else
                        *reinterpret_cast<uint4*>(dst) = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]),
                                                                    pack2(f[4], f[5]), pack2(f[6], f[7]));
                    if constexpr (SPLIT)
                        *reinterpret_cast<uint4*>(dst + 2 * TILE) =
                            make_uint4(pack2(lo_part(f[0]), lo_part(f[1])), pack2(lo_part(f[2]), lo_part(f[3])),
                                       pack2(lo_part(f[4]), lo_part(f[5])), pack2(lo_part(f[6]), lo_part(f[7])));
                }
                l_run = l_run * alpha + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
                m_run = m_new;
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full + (g & 1));
            }
            // the row sum over both halves (every softmax thread reaches this barrier, aborted or not)
            red[half * BQ + row] = l_run;
            named_bar_sync(1, 256);
            const float l_all = red[row] + red[BQ + row];
            named_bar_sync(1, 256);   // both halves have read the sums before the next item's maxima overwrite them
            const uint32_t last = base + nk - 1;
            ok = __all_sync(0xffffffffu, ok && mbar_wait(o_done + (last & 1), (last >> 1) & 1, abort_flag, p.err));
            if (ok) {
                tc_fence_after();
                const float inv = l_all > 0.f ? 1.0f / l_all : 0.f;
                uint32_t o[HO];
                tmem_ld32(tO + lane_off + half * HO, o);
                tmem_ld_wait();
                // O is in registers: the next item's first P·V may overwrite it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(o_free);
                if (Q8OUT && q < L) {
                    float f[HO];
                    float m = 0.f;
#pragma unroll
                    for (int e = 0; e < HO; ++e) {
                        f[e] = __uint_as_float(o[e]) * inv;
                        m = fmaxf(m, fabsf(f[e]));
                    }
                    const float id = m != 0.0f ? __fdiv_rn(127.0f, m) : 0.0f;
                    const size_t tok = static_cast<size_t>(seg0 + q);
                    __half* qrow = p.q8 + tok * p.hidden + head * HD + half * HO;
#pragma unroll
                    for (int t = 0; t < HO / 8; ++t) {
                        __half hq[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) hq[e] = __int2half_rn(__float2int_rn(__fmul_rn(f[8 * t + e], id)));
                        *reinterpret_cast<uint4*>(qrow + 8 * t) = *reinterpret_cast<const uint4*>(hq);
                    }
                    p.q8d[static_cast<size_t>(head * 2 + half) * p.q8ldd + tok] = round_fp16(__fdiv_rn(m, 127.0f));
                } else if (q < L) {
                    __nv_bfloat16* orow = p.out + static_cast<size_t>(seg0 + q) * p.ldo + head * HD + half * HO;
#pragma unroll
                    for (int t = 0; t < HO / 8; ++t) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[8 * t + e]) * inv;
                        *reinterpret_cast<uint4*>(orow + 8 * t) =
                            make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                        if constexpr (HILO) {
                            __nv_bfloat16* lrow = p.out_lo + static_cast<size_t>(seg0 + q) * p.ldo + head * HD + half * HO;
                            *reinterpret_cast<uint4*>(lrow + 8 * t) =
                                make_uint4(pack2(lo_part(f[0]), lo_part(f[1])), pack2(lo_part(f[2]), lo_part(f[3])),
                                           pack2(lo_part(f[4]), lo_part(f[5])), pack2(lo_part(f[6]), lo_part(f[7])));
                        }
                    }
                    if (!INFER && half == 0) p.lse[static_cast<size_t>(seg0 + q) * p.heads + head] = m_run + logf(l_all);
                }
            }
            base += nk;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}


// ------------------------------------------------------------------------------------------------ backward: dK, dV
// Same contract as fa::bwd_dkdv_kernel (flash.cu; Ops.AttentionBackward, Laya.Training/Ops.cs:368-470): for one
// 128-key tile of one head, over every 64-query tile that sees it,
//     Sᵀ = K·Qᵀ,  dPᵀ = V·dOᵀ  (M 128 keys, N 64 queries, K 64)            into TMEM columns [0, 64), [64, 128)
//     Pᵀ = exp(scale·Sᵀ − lse) (· dropout),  dSᵀ = P ∘ (scale·dPᵀ·m − scale·D)   by the softmax warps
//     dV += Pᵀ·dO,  dK += dSᵀ·Q  (M 128 keys, N 64, K 64 queries; dO and Q read N-contiguous) into [128, 256)
// then dK (rotated back by −θ at the key's position) and dV in bf16.  Pᵀ goes back into the TMEM columns of dPᵀ it was
// formed from (bf16 pairs, queries [0, 32) at [64, 80) and [32, 64) at [96, 112): each thread overwrites only columns
// it has already read) and is the A operand of the dV MMA read from tensor memory; dSᵀ goes to shared memory (the A
// operand of dK, and the tile the dQ kernel reads from the scratch).  With Pᵀ out of shared memory a CTA holds K, V,
// three (Q, dO) stages and dSᵀ in ~99 KB, so two CTAs share an SM.  MMA order per tile j: Sᵀ(j) as soon as the
// softmax has read Sᵀ(j − 1); then, once the softmax has finished tile j − 1, dV(j − 1), dK(j − 1) and dPᵀ(j) (dPᵀ(j)
// overwrites Pᵀ(j − 1) after the dV MMA that reads it: MMAs of one thread run in order).  The softmax of tile j forms
// P from Sᵀ(j) while dV/dK(j − 1) and dPᵀ(j) run.  lse and D of a query tile are staged next to its Q and dO tiles by
// the producer warp, read from HBM before the producer waits for the stage; with precomputed dropout decisions
// (BwdParams::dmask) so are the tile's four words per query, from which each softmax thread takes its key's bits.
struct BwdParams {
    const int32_t* seg_start; const int32_t* seg_len;
    const int32_t* tq_item; const int32_t* tq_p0; const int32_t* n_tq;
    int window, hidden, heads;
    float scale, dropout, keep;
    uint64_t seed;
    const float* lse; const float* dsum;
    const float* cosv; const float* sinv;
    __nv_bfloat16* dqkv; int lddq;
    int* err;
    uint8_t* ds; int ds_nq;   // the dS scratch (fa::Args) or null
    int wave;                 // dK/dV: CTAs resident at once (two per SM)
    const uint32_t* dmask; int dmask_w, dmask_rows;   // precomputed dropout decisions (fa::Args), or null
};
constexpr int BQ2 = 64;                          // queries per tile of the dK/dV kernel
constexpr int QTILE2 = BQ2 * 128;                // bytes of one 64-row × 64-column bf16 tile
constexpr int BWD_ST = 3;                        // (Q, dO) stages
constexpr int BWD_MW = BK / 32;                  // dropout-decision words per query row of a key tile
constexpr int BWD_SMEM = 1024 + 2 * TILE + BWD_ST * 2 * QTILE2 + TILE + BWD_ST * 2 * BQ2 * 4 +
                         BWD_ST * BWD_MW * BQ2 * 4 + 256;   // K, V, stages, dSᵀ; lse/D; dropout words
static_assert(2 * BWD_SMEM <= 232448, "two CTAs per SM");

DEVI void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
DEVI void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
// D[tmem] (+)= A[tmem] · B[smem] (kind::f16): A is M 128 rows in the TMEM lanes × K 16, two 16-bit values per column.
DEVI void mma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <bool DROP>
__global__ void __launch_bounds__(320, 2)
    bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmq,
                       const __grid_constant__ CUtensorMap tmdo, BwdParams p) {
    constexpr uint32_t IDESC_S = make_idesc(1, 1, 1, BK, BQ2);                    // M keys, N queries, K-major
    constexpr uint32_t IDESC_G = make_idesc(1, 1, 1, BK, HD) | (1u << 16);        // B (dO, Q) N-contiguous
    const int tile = blockIdx.x, n_tq = *p.n_tq;
    if (tile >= n_tq) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sK = smem;
    uint8_t* sV = smem + TILE;
    uint8_t* sQO = smem + 2 * TILE;              // [BWD_ST stages][Q, dO], 64 rows each
    uint8_t* sDS = sQO + BWD_ST * 2 * QTILE2;    // dSᵀ [128 keys × 64 queries]
    float* sRow = reinterpret_cast<float*>(sDS + TILE);   // [BWD_ST stages][−lse·log2 e 64 | −scale·D 64]
    uint32_t* sMask = reinterpret_cast<uint32_t*>(sRow + BWD_ST * 2 * BQ2);   // [BWD_ST][word 4][query 64] (DROP)
    uint64_t* bars = reinterpret_cast<uint64_t*>(sMask + BWD_ST * BWD_MW * BQ2);
    uint64_t* kv_full = bars;
    uint64_t* full = bars + 1;                   // [BWD_ST]
    uint64_t* empty = bars + 1 + BWD_ST;         // [BWD_ST]
    uint64_t* s_full = bars + 1 + 2 * BWD_ST;    // Sᵀ(j) in TMEM
    uint64_t* s_free = s_full + 1;               // Sᵀ(j) read by the softmax
    uint64_t* dp_full = s_full + 2;              // dPᵀ(j) in TMEM
    uint64_t* pd_full = s_full + 3;              // Pᵀ(j) in TMEM, dSᵀ(j) in smem
    uint64_t* pd_empty = s_full + 4;             // dSᵀ(j) read by its dK MMA and its scratch copy
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int head = blockIdx.y, item = p.tq_item[tile], k0 = p.tq_p0[tile];
    const int seg0 = p.seg_start[item], L = p.seg_len[item];
    const bool global = p.window < 0;
    const int W = p.window;
    const int qb0 = global ? 0 : max(0, k0 - W), qe = global ? L : min(L, k0 + BK + W);
    const int nq = (qe - qb0 + BQ2 - 1) / BQ2;
    const int warp = warp_id(), lane = lane_id();

    if (threadIdx.x == 0) {
        mbar_init(kv_full, 1);
        for (int s = 0; s < BWD_ST; ++s) { mbar_init(full + s, 2); mbar_init(empty + s, 1); }
        mbar_init(s_full, 1);
        mbar_init(s_free, 8);
        mbar_init(dp_full, 1);
        mbar_init(pd_full, 8);
        mbar_init(pd_empty, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 256); tmem_relinquish(); }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmk); prefetch_tmap(&tmq); prefetch_tmap(&tmdo); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tDP = tmem + BQ2, tDV = tmem + 2 * BQ2, tDK = tmem + 2 * BQ2 + HD;

    if (warp == 0) {
        // ---- producer: K and V once; per query tile Q and dO by TMA, lse and D by the warp's lanes
        if (lane == 0) {
            mbar_arrive_expect_tx(kv_full, 2 * TILE);
            tma_load_2d(sK, &tmk, kv_full, p.hidden + head * HD, seg0 + k0);
            tma_load_2d(sV, &tmk, kv_full, 2 * p.hidden + head * HD, seg0 + k0);
        }
        for (int j = 0; j < nq; ++j) {
            const int s = j % BWD_ST;
            const int q0 = qb0 + j * BQ2;
            // the tile's row statistics are read before the wait for its stage, so their latency overlaps it; they
            // are staged as the softmax uses them: −lse·log2(e) and −scale·D
            float lv[BQ2 / 32], dv[BQ2 / 32];
#pragma unroll
            for (int i = 0; i < BQ2 / 32; ++i) {
                const int r = lane + 32 * i;
                const bool in = q0 + r < qe;
                const size_t at = static_cast<size_t>(seg0 + (in ? q0 + r : 0)) * p.heads + head;
                lv[i] = in ? -__ldg(p.lse + at) * LOG2E : 0.f;
                dv[i] = in ? -p.scale * __ldg(p.dsum + at) : 0.f;
            }
            uint4 mw[BQ2 / 32];   // DROP with precomputed decisions: each of the lane's queries' 4 words of this key tile
            if (DROP && p.dmask) {
#pragma unroll
                for (int i = 0; i < BQ2 / 32; ++i) {
                    const int q = q0 + lane + 32 * i;
                    mw[i] = q < qe ? __ldg(reinterpret_cast<const uint4*>(
                                         p.dmask + (static_cast<size_t>(head) * p.dmask_rows + seg0 + q) * p.dmask_w + k0 / 32))
                                   : make_uint4(0u, 0u, 0u, 0u);
                }
            }
            int got = 1;
            if (lane == 0) got = mbar_wait(empty + s, ((j / BWD_ST) & 1) ^ 1, abort_flag, p.err);
            if (!__shfl_sync(0xffffffffu, got, 0)) break;
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(full + s, 2 * QTILE2);
                tma_load_2d(sQO + s * 2 * QTILE2, &tmq, full + s, head * HD, seg0 + q0);
                tma_load_2d(sQO + s * 2 * QTILE2 + QTILE2, &tmdo, full + s, head * HD, seg0 + q0);
            }
            float* rows = sRow + s * 2 * BQ2;
#pragma unroll
            for (int i = 0; i < BQ2 / 32; ++i) {
                rows[lane + 32 * i] = lv[i];
                rows[BQ2 + lane + 32 * i] = dv[i];
            }
            if (DROP && p.dmask) {
                uint32_t* mrow = sMask + s * BWD_MW * BQ2;
#pragma unroll
                for (int i = 0; i < BQ2 / 32; ++i) {
                    const int r = lane + 32 * i;
                    mrow[0 * BQ2 + r] = mw[i].x;
                    mrow[1 * BQ2 + r] = mw[i].y;
                    mrow[2 * BQ2 + r] = mw[i].z;
                    mrow[3 * BQ2 + r] = mw[i].w;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(full + s);
        }
    } else if (warp == 1) {
        // ---- MMA issuer.  Iteration j: Sᵀ(j); the deferred release of dSᵀ(j − 2); dV/dK(j − 1); dPᵀ(j).
        if (lane == 0) {
            bool ok = mbar_wait(kv_full, 0, abort_flag, p.err);
            tc_fence_after();
            const uint32_t ak = smem_u32(sK), av = smem_u32(sV), ad = smem_u32(sDS);
            bool pend = false;   // a dSᵀ tile whose scratch copy and dK MMA must finish reading before pd_empty
            for (int j = 0; j <= nq && ok; ++j) {
                const int s = j % BWD_ST;
                const uint32_t aq = smem_u32(sQO + s * 2 * QTILE2), ado = aq + QTILE2;
                if (j < nq) {
                    if (!mbar_wait(full + s, (j / BWD_ST) & 1, abort_flag, p.err)) { ok = false; break; }
                    if (j > 0 && !mbar_wait(s_free, (j - 1) & 1, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        mma_f16(tS, smem_desc_sw128(ak + kk * 32), smem_desc_sw128(aq + kk * 32), IDESC_S, kk > 0);
                    mma_commit(s_full);
                }
                if (pend) {   // by now the copy has long read its tile: no wait in the common case
                    if (p.ds) bulk_wait_read_all();
                    mma_commit(pd_empty);
                    pend = false;
                }
                if (j >= 1) {
                    const int i = j - 1, si = i % BWD_ST;
                    if (!mbar_wait(pd_full, i & 1, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t aqi = smem_u32(sQO + si * 2 * QTILE2), adoi = aqi + QTILE2;
                    if (p.ds) {   // dSᵀ of tile i to the scratch for dQ = dS·K, its read overlapping the MMAs
                        const size_t idx = 1 + (static_cast<size_t>(tile) * p.ds_nq + i) * p.heads + head;
                        bulk_store(p.ds + idx * TILE, sDS, TILE);
                        bulk_commit();
                    }
#pragma unroll
                    for (int kk = 0; kk < BQ2 / 16; ++kk) {
                        const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                        // Pᵀ queries [16kk, 16kk + 16) sit at dPᵀ column 8kk, +16 for the second half-row
                        mma_ts_f16(tDV, tDP + static_cast<uint32_t>(kk * 8 + (kk >= 2 ? 16 : 0)),
                                   desc_mn_sw128(adoi + kk * 2048, QTILE2), IDESC_G, acc);
                        mma_f16(tDK, smem_desc_sw128(ad + kk * 32), desc_mn_sw128(aqi + kk * 2048, QTILE2), IDESC_G, acc);
                    }
                    mma_commit(empty + si);
                    pend = true;
                }
                if (j < nq) {   // dPᵀ(j) over Pᵀ(j − 1): issued after the dV MMA that reads it
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        mma_f16(tDP, smem_desc_sw128(av + kk * 32), smem_desc_sw128(ado + kk * 32), IDESC_S, kk > 0);
                    mma_commit(dp_full);
                }
            }
            if (pend && ok) {
                if (p.ds) bulk_wait_read_all();
                mma_commit(pd_empty);
            }
            if (p.ds) bulk_wait_all();
        } else if (lane == 1 && p.wave > 0) {
            // warm L2 with the K and V tiles of the CTA one resident wave ahead in launch order, whose first loads
            // would otherwise come from DRAM after it starts
            const long long lin = static_cast<long long>(blockIdx.y) * gridDim.x + blockIdx.x + p.wave;
            const int t2 = static_cast<int>(lin % gridDim.x), h2 = static_cast<int>(lin / gridDim.x);
            if (h2 < p.heads && t2 < n_tq) {
                const int y2 = p.seg_start[p.tq_item[t2]] + p.tq_p0[t2];
                tma_prefetch_2d(&tmk, p.hidden + h2 * HD, y2);
                tma_prefetch_2d(&tmk, 2 * p.hidden + h2 * HD, y2);
            }
        }
    } else {
        // ---- softmax warps: thread (half, row) owns key row `row` and queries [32·half, 32·half + 32) of a tile
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const int key = k0 + row;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        constexpr int HQ = BQ2 / 2;
        const float sl2 = p.scale * LOG2E;
        const uint64_t sl2x2 = f2_pack(sl2, sl2), scale2 = f2_pack(p.scale, p.scale);
        // the queries this key sees: [vlo, vhi] (within the tile's query range [qb0, qe) by construction)
        const bool kin = key < L;
        const int vlo = global ? 0 : key - W;
        const int vhi = global ? L - 1 : min(L - 1, key + W);
        uint8_t* drow = sDS + row * 128;
        const uint32_t tSh = tS + lane_off + half * HQ, tDPh = tDP + lane_off + half * HQ;
        bool ok = true;
        for (int j = 0; j < nq; ++j) {
            const int s = j % BWD_ST;
            ok = __all_sync(0xffffffffu, ok && mbar_wait(s_full, j & 1, abort_flag, p.err) &&
                                             mbar_wait(full + s, (j / BWD_ST) & 1, abort_flag, p.err));
            const float* rows = sRow + s * 2 * BQ2 + half * HQ;
            const int q0 = qb0 + j * BQ2 + half * HQ;
            // P = 2^(S·scale·log2 e − lse·log2 e) for the half-row's 32 queries, two per .f32x2 instruction; a masked
            // pair member gets the exponent −inf (P = 0).  The row statistics are the same for every thread
            // (broadcast four-wide reads).
            uint32_t pv[32];
            if (ok) {
                tc_fence_after();
                tmem_ld16(tSh, *reinterpret_cast<uint32_t(*)[16]>(pv));
                tmem_ld16(tSh + 16, *reinterpret_cast<uint32_t(*)[16]>(pv + 16));
                tmem_ld_wait();
            }
            tc_fence_before();   // Sᵀ is in registers: release it to the next tile's MMA
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            if (!ok) continue;
            const bool whole = __all_sync(0xffffffffu, kin && q0 >= vlo && q0 + HQ - 1 <= vhi);
            uint32_t kept = 0xffffffffu;   // dropout: which of the 32 probabilities are kept
            if (DROP && p.dmask) {   // this key's bit (lane) of the half-row's 32 queries' words (quarter)
                const uint4* w4 = reinterpret_cast<const uint4*>(sMask + s * BWD_MW * BQ2 + quarter * BQ2 + half * HQ);
                kept = 0u;
#pragma unroll
                for (int t = 0; t < HQ / 4; ++t) {
                    const uint4 w = w4[t];
                    kept |= (((w.x >> lane) & 1u) << (4 * t)) | (((w.y >> lane) & 1u) << (4 * t + 1)) |
                            (((w.z >> lane) & 1u) << (4 * t + 2)) | (((w.w >> lane) & 1u) << (4 * t + 3));
                }
            }
            {
                fat::DropWalk walk(p.seed, head, seg0 + q0, key, 1ull << 21, p.dropout, p.keep);
                const float4* nl4 = reinterpret_cast<const float4*>(rows);
#pragma unroll
                for (int t = 0; t < HQ / 4; ++t) {
                    const float4 nl = nl4[t];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int e = 4 * t + 2 * u;
                        float a0, a1;
                        f2_unpack(f2_fma(f2_pack(__uint_as_float(pv[e]), __uint_as_float(pv[e + 1])), sl2x2,
                                         u ? f2_pack(nl.z, nl.w) : f2_pack(nl.x, nl.y)),
                                  a0, a1);
                        if (!whole) {
                            const int q = q0 + e;
                            if (!(kin && q >= vlo && q <= vhi)) a0 = -INFINITY;
                            if (!(kin && q + 1 >= vlo && q + 1 <= vhi)) a1 = -INFINITY;
                        }
                        pv[e] = __float_as_uint(ex2(a0));
                        pv[e + 1] = __float_as_uint(ex2(a1));
                        if constexpr (DROP) {
                            if (!p.dmask) {
                                if (walk.next() == 0.f) kept &= ~(1u << e);
                                if (walk.next() == 0.f) kept &= ~(1u << (e + 1));
                            }
                        }
                    }
                }
            }
            // dSᵀ = P ∘ (scale·dPᵀ·m − scale·D) in 16-query pieces; Pᵀ·m back over the dPᵀ columns just read
            ok = __all_sync(0xffffffffu, mbar_wait(dp_full, j & 1, abort_flag, p.err));
            if (!ok) continue;
            uint32_t dall[32];   // the half-row's dPᵀ in one TMEM round trip
            tc_fence_after();
            tmem_ld16(tDPh, *reinterpret_cast<uint32_t(*)[16]>(dall));
            tmem_ld16(tDPh + 16, *reinterpret_cast<uint32_t(*)[16]>(dall + 16));
            tmem_ld_wait();
            // dSᵀ of the previous tile must have been read by its dK MMA and its scratch copy before it is rewritten
            if (j > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(pd_empty, (j - 1) & 1, abort_flag, p.err));
                if (!ok) continue;
            }
#pragma unroll
            for (int pc = 0; pc < 2; ++pc) {
                uint32_t* dv = dall + pc * 16;
                const float4* sd4 = reinterpret_cast<const float4*>(rows + BQ2 + pc * 16);
                uint32_t pk[8];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float4 sd = sd4[t];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int e = 4 * t + 2 * u, ep = pc * 16 + e;
                        const float pe0 = __uint_as_float(pv[ep]), pe1 = __uint_as_float(pv[ep + 1]);
                        float d0 = __uint_as_float(dv[e]), d1 = __uint_as_float(dv[e + 1]);
                        float p0 = pe0, p1 = pe1;
                        if constexpr (DROP) {
                            const float m0 = (kept >> ep) & 1u ? p.keep : 0.f, m1 = (kept >> (ep + 1)) & 1u ? p.keep : 0.f;
                            p0 *= m0; p1 *= m1;
                            d0 *= m0; d1 *= m1;
                        }
                        float g0, g1;
                        f2_unpack(f2_mul(f2_pack(pe0, pe1),
                                         f2_fma(scale2, f2_pack(d0, d1), u ? f2_pack(sd.z, sd.w) : f2_pack(sd.x, sd.y))),
                                  g0, g1);
                        pk[e / 2] = pack2(p0, p1);
                        dv[e] = __float_as_uint(g0);
                        dv[e + 1] = __float_as_uint(g1);
                    }
                }
                tmem_st8(tDP + lane_off + static_cast<uint32_t>(half * HQ + pc * 8), pk);
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const float* g = reinterpret_cast<const float*>(dv + 8 * u);
                    const int off = ((half * 4 + pc * 2 + u) ^ (row & 7)) << 4;
                    *reinterpret_cast<uint4*>(drow + off) =
                        make_uint4(pack2(g[0], g[1]), pack2(g[2], g[3]), pack2(g[4], g[5]), pack2(g[6], g[7]));
                }
            }
            tmem_st_wait();
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(pd_full);
        }
        // dK (half 0, rotated back by −θ, pairs (i, i + 32) sixteen at a time) and dV (half 1, 32 columns at a time)
        // once the last dV/dK MMAs are done
        ok = __all_sync(0xffffffffu, ok && nq > 0 && mbar_wait(pd_empty, (nq - 1) & 1, abort_flag, p.err));
        if (ok) {
            tc_fence_after();
            __nv_bfloat16* out = p.dqkv + static_cast<size_t>(seg0 + key) * p.lddq + (half == 0 ? p.hidden : 2 * p.hidden) + head * HD;
            if (half == 0) {
#pragma unroll 1
                for (int pc = 0; pc < 2; ++pc) {
                    uint32_t x[16], y[16];
                    tmem_ld16(tDK + lane_off + pc * 16, x);
                    tmem_ld16(tDK + lane_off + 32 + pc * 16, y);
                    tmem_ld_wait();
                    if (key < L) {
                        float a[16], b[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            a[e] = __uint_as_float(x[e]);
                            b[e] = __uint_as_float(y[e]);
                        }
                        if (p.cosv) {   // 16-byte aligned tables (checked at launch): four-wide loads
                            const float4* c4 = reinterpret_cast<const float4*>(p.cosv + static_cast<size_t>(key) * (HD / 2) + pc * 16);
                            const float4* s4 = reinterpret_cast<const float4*>(p.sinv + static_cast<size_t>(key) * (HD / 2) + pc * 16);
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const float4 c = __ldg(c4 + t), sn = __ldg(s4 + t);
                                const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
                                for (int u4 = 0; u4 < 4; ++u4) {
                                    const int e = 4 * t + u4;
                                    const float u = a[e], v = b[e];
                                    a[e] = __fadd_rn(__fmul_rn(u, cc[u4]), __fmul_rn(v, ss[u4]));
                                    b[e] = __fsub_rn(__fmul_rn(v, cc[u4]), __fmul_rn(u, ss[u4]));
                                }
                            }
                        }
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            *reinterpret_cast<uint4*>(out + pc * 16 + 8 * t) =
                                make_uint4(pack2(a[8 * t], a[8 * t + 1]), pack2(a[8 * t + 2], a[8 * t + 3]),
                                           pack2(a[8 * t + 4], a[8 * t + 5]), pack2(a[8 * t + 6], a[8 * t + 7]));
                            *reinterpret_cast<uint4*>(out + 32 + pc * 16 + 8 * t) =
                                make_uint4(pack2(b[8 * t], b[8 * t + 1]), pack2(b[8 * t + 2], b[8 * t + 3]),
                                           pack2(b[8 * t + 4], b[8 * t + 5]), pack2(b[8 * t + 6], b[8 * t + 7]));
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int pc = 0; pc < 2; ++pc) {
                    uint32_t x[32];
                    tmem_ld32(tDV + lane_off + pc * 32, x);
                    tmem_ld_wait();
                    if (key < L) {
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float* f = reinterpret_cast<const float*>(x + 8 * t);
                            *reinterpret_cast<uint4*>(out + pc * 32 + 8 * t) =
                                make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ------------------------------------------------------------------------------------------------ backward: dQ
// Same contract as fa::bwd_dq_kernel (flash.cu): for one 128-query tile of one head, over every 64-key tile it sees,
//     S = Q·Kᵀ,  dP = dO·Vᵀ  (M 128 queries, N 64 keys, K 64)                into TMEM columns [0, 64), [64, 128)
//     P = exp(scale·S − lse) (· dropout),  dS = scale · P ∘ (dP·m − D)       by the softmax warps, bf16 into smem
//     dQ += dS·K  (M 128 queries, N 64, K 64 keys; K read N-contiguous)      into [128, 192)
// then dQ rotated back by −θ at the query's position, in bf16.  Roles as in the forward: warp 0 loads Q and dO once
// and K, V through a 2-stage ring; warp 1 issues the MMAs (S and dP of tile j before dQ of tile j − 1); warps 2-9
// are the softmax warps, thread (half, row) owning query row `row` and keys [32·half, 32·half + 32) of a tile.
// 64-key tiles keep a CTA within 256 TMEM columns and 82 KB of shared memory, so two CTAs share an SM and one's
// MMA round trips overlap the other's softmax (a sliding-window tile sees only a few key tiles).
constexpr int DQ_BK = 64;
constexpr int DQ_KTILE = DQ_BK * 128;                        // bytes of one 64-key × 64-column bf16 tile
constexpr int DQ_SMEM = 1024 + 2 * TILE + 4 * DQ_KTILE + TILE + 256;   // Q, dO, 2 × (K, V), dS; barriers
static_assert(2 * DQ_SMEM <= 232448, "two CTAs per SM");


// Persistent like the forward: a CTA walks (query tile, head) items and every barrier phase runs on across items.
template <bool DROP>
__global__ void __launch_bounds__(320, 2)
    bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv,
                     const __grid_constant__ CUtensorMap tmdo, BwdParams p) {
    constexpr uint32_t IDESC_S = make_idesc(1, 1, 1, BQ, DQ_BK);                  // M queries, N keys, K-major
    constexpr uint32_t IDESC_G = make_idesc(1, 1, 1, BQ, HD) | (1u << 16);        // B (K) N-contiguous
    const int n_items = *p.n_tq * p.heads;
    if (static_cast<int>(blockIdx.x) >= n_items) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sDO = smem + TILE;
    uint8_t* sKV = smem + 2 * TILE;                 // [2 stages][K, V], 64 keys each
    uint8_t* sDS = sKV + 4 * DQ_KTILE;              // dS [128 queries × 64 keys]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + TILE);
    uint64_t* qo_full = bars;
    uint64_t* kv_full = bars + 1;     // [2]
    uint64_t* kv_empty = bars + 3;    // [2]
    uint64_t* st_full = bars + 5;
    uint64_t* st_free = bars + 6;
    uint64_t* ds_full = bars + 7;
    uint64_t* ds_empty = bars + 8;
    uint64_t* qo_empty = bars + 9;    // Q and dO read by the item's last S and dP MMAs
    uint64_t* dq_free = bars + 10;    // dQ read by the item's epilogue
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const bool global = p.window < 0;
    const int W = p.window;
    const int warp = warp_id(), lane = lane_id();
    auto span_of = [&](int item, int& head, int& seg0, int& L, int& q0, int& kb, int& nk) {
        const int tile = item / p.heads;
        head = item - tile * p.heads;
        const int it = p.tq_item[tile];
        q0 = p.tq_p0[tile];
        seg0 = p.seg_start[it];
        L = p.seg_len[it];
        kb = global ? 0 : max(0, q0 - W);
        const int ke = global ? L : min(L, q0 + BQ + W);
        nk = (ke - kb + DQ_BK - 1) / DQ_BK;
    };

    if (threadIdx.x == 0) {
        mbar_init(qo_full, 1);
        mbar_init(qo_empty, 1);
        mbar_init(dq_free, 8);
        for (int s = 0; s < 2; ++s) { mbar_init(kv_full + s, 1); mbar_init(kv_empty + s, 1); }
        mbar_init(st_full, 1);
        mbar_init(st_free, 8);
        mbar_init(ds_full, 8);
        mbar_init(ds_empty, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 256); tmem_relinquish(); }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmq); prefetch_tmap(&tmkv); prefetch_tmap(&tmdo); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem, tDP = tmem + DQ_BK, tDQ = tmem + 2 * DQ_BK;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0, n = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
                int head, seg0, L, q0, kb, nk;
                span_of(item, head, seg0, L, q0, kb, nk);
                if (!mbar_wait(qo_empty, (n & 1) ^ 1, abort_flag, p.err)) break;
                mbar_arrive_expect_tx(qo_full, 2 * TILE);
                tma_load_2d(sQ, &tmq, qo_full, head * HD, seg0 + q0);
                tma_load_2d(sDO, &tmdo, qo_full, head * HD, seg0 + q0);
                for (int j = 0; j < nk; ++j, ++g) {
                    const int s = g & 1;
                    if (!mbar_wait(kv_empty + s, ((g >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    uint8_t* st = sKV + s * 2 * DQ_KTILE;
                    const int y = seg0 + kb + j * DQ_BK;
                    mbar_arrive_expect_tx(kv_full + s, 2 * DQ_KTILE);
                    tma_load_2d(st, &tmkv, kv_full + s, p.hidden + head * HD, y);
                    tma_load_2d(st + DQ_KTILE, &tmkv, kv_full + s, 2 * p.hidden + head * HD, y);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t base = 0, n = 0;
            bool ok = true;
            const uint32_t aq = smem_u32(sQ), ado = smem_u32(sDO);
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++n) {
                int head, seg0, L, q0, kb, nk;
                span_of(item, head, seg0, L, q0, kb, nk);
                if (!mbar_wait(qo_full, n & 1, abort_flag, p.err)) break;
                tc_fence_after();
                for (int j = 0; j <= nk; ++j) {
                    if (j < nk) {
                        const uint32_t g = base + j;
                        const int s = g & 1;
                        if (!mbar_wait(kv_full + s, (g >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
                        // S and dP of the previous tile (of this item or the last) must have been read
                        if (g > 0 && !mbar_wait(st_free, (g - 1) & 1, abort_flag, p.err)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t ak = smem_u32(sKV + s * 2 * DQ_KTILE), av = ak + DQ_KTILE;
#pragma unroll
                        for (int kk = 0; kk < HD / 16; ++kk) {
                            mma_f16(tS, smem_desc_sw128(aq + kk * 32), smem_desc_sw128(ak + kk * 32), IDESC_S, kk > 0);
                            mma_f16(tDP, smem_desc_sw128(ado + kk * 32), smem_desc_sw128(av + kk * 32), IDESC_S, kk > 0);
                        }
                        mma_commit(st_full);
                        if (j == nk - 1) mma_commit(qo_empty);
                    }
                    if (j >= 1) {
                        const int i = j - 1;
                        const uint32_t gi = base + i;
                        const int s = gi & 1;
                        if (!mbar_wait(ds_full, gi & 1, abort_flag, p.err)) { ok = false; break; }
                        // the item's first dQ MMA overwrites dQ: the previous item's epilogue must have read it
                        if (i == 0 && !mbar_wait(dq_free, (n & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t ak = smem_u32(sKV + s * 2 * DQ_KTILE), ads = smem_u32(sDS);
#pragma unroll
                        for (int kk = 0; kk < DQ_BK / 16; ++kk)
                            mma_f16(tDQ, smem_desc_sw128(ads + kk * 32), desc_mn_sw128(ak + kk * 2048, DQ_KTILE), IDESC_G,
                                    (i > 0 || kk > 0) ? 1u : 0u);
                        mma_commit(kv_empty + s);
                        mma_commit(ds_empty);
                    }
                }
                base += nk;
            }
        }
    } else {
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        constexpr int HK = DQ_BK / 2;
        const float sl2 = p.scale * LOG2E;
        uint8_t* drow = sDS + row * 128;
        bool ok = true;
        uint32_t base = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            int head, seg0, L, q0, kb, nk;
            span_of(item, head, seg0, L, q0, kb, nk);
            const int q = q0 + row;
            const bool qin = q < L;
            const size_t at = static_cast<size_t>(seg0 + (qin ? q : 0)) * p.heads + head;
            const float lse2 = qin ? __ldg(p.lse + at) * LOG2E : 0.f, dd = qin ? __ldg(p.dsum + at) : 0.f;
            // keys this row sees: [lo, lo + span]
            const int lo = global ? 0 : max(0, q - W);
            const int span = (global ? L - 1 : min(L - 1, q + W)) - lo;
            for (int j = 0; j < nk; ++j) {
                const uint32_t g = base + j;
                ok = __all_sync(0xffffffffu, ok && mbar_wait(st_full, g & 1, abort_flag, p.err));
                const int k0 = kb + j * DQ_BK + half * HK;
                DropWalk walk(p.seed, head, seg0 + q, k0, 1, p.dropout, p.keep);
                // the half-row's 32 keys in two 16-key pieces (fewer live registers): read S and dP, form dS, store it
#pragma unroll
                for (int pc = 0; pc < 2; ++pc) {
                    uint32_t sv[16], dv[16];
                    if (ok) {
                        tc_fence_after();
                        tmem_ld16(tS + lane_off + half * HK + pc * 16, sv);
                        tmem_ld16(tDP + lane_off + half * HK + pc * 16, dv);
                        tmem_ld_wait();
                    }
                    if (pc == 1) {   // S and dP are in registers: release them to the next tile's MMAs
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(st_free);
                    }
                    if (!ok) continue;
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int k = k0 + pc * 16 + e;
                        const bool vis = qin && static_cast<unsigned>(k - lo) <= static_cast<unsigned>(span);
                        const float pe = vis ? ex2(fmaf(__uint_as_float(sv[e]), sl2, -lse2)) : 0.f;
                        const float m = DROP ? walk.next() : 1.0f;
                        sv[e] = __float_as_uint(p.scale * pe * (__uint_as_float(dv[e]) * m - dd));
                    }
                    // dS of the previous tile must have been read by its dQ MMAs before it is rewritten
                    if (pc == 0 && g > 0) {
                        ok = __all_sync(0xffffffffu, mbar_wait(ds_empty, (g - 1) & 1, abort_flag, p.err));
                        if (!ok) continue;
                    }
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const float* f = reinterpret_cast<const float*>(sv + 8 * u);
                        *reinterpret_cast<uint4*>(drow + (((half * 4 + pc * 2 + u) ^ (row & 7)) << 4)) =
                            make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                    }
                }
                if (!ok) continue;
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(ds_full);
            }
            // dQ once the item's last dQ MMAs are done: half h rotates the pairs (i, i + 32) for i in [16h, 16h + 16)
            // back by −θ and stores them
            const uint32_t last = base + nk - 1;
            ok = __all_sync(0xffffffffu, ok && nk > 0 && mbar_wait(ds_empty, last & 1, abort_flag, p.err));
            if (ok) {
                tc_fence_after();
                uint32_t x[16], y[16];
                tmem_ld16(tDQ + lane_off + half * 16, x);
                tmem_ld16(tDQ + lane_off + 32 + half * 16, y);
                tmem_ld_wait();
                // dQ is in registers: the next item's first dQ MMA may overwrite it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(dq_free);
                if (qin) {
                    float a[16], b[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        a[e] = __uint_as_float(x[e]);
                        b[e] = __uint_as_float(y[e]);
                    }
                    if (p.cosv) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const int i = half * 16 + e;
                            const float c = p.cosv[static_cast<size_t>(q) * (HD / 2) + i];
                            const float sn = p.sinv[static_cast<size_t>(q) * (HD / 2) + i];
                            const float u = a[e], v = b[e];
                            a[e] = __fadd_rn(__fmul_rn(u, c), __fmul_rn(v, sn));
                            b[e] = __fsub_rn(__fmul_rn(v, c), __fmul_rn(u, sn));
                        }
                    }
                    __nv_bfloat16* out = p.dqkv + static_cast<size_t>(seg0 + q) * p.lddq + head * HD + half * 16;
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        *reinterpret_cast<uint4*>(out + 8 * t) =
                            make_uint4(pack2(a[8 * t], a[8 * t + 1]), pack2(a[8 * t + 2], a[8 * t + 3]),
                                       pack2(a[8 * t + 4], a[8 * t + 5]), pack2(a[8 * t + 6], a[8 * t + 7]));
                        *reinterpret_cast<uint4*>(out + 32 + 8 * t) =
                            make_uint4(pack2(b[8 * t], b[8 * t + 1]), pack2(b[8 * t + 2], b[8 * t + 3]),
                                       pack2(b[8 * t + 4], b[8 * t + 5]), pack2(b[8 * t + 6], b[8 * t + 7]));
                    }
                }
            }
            base += nk;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ------------------------------------------------------------------------------------------------ backward: dQ = dS·K
// dQ from the dSᵀ tiles the dK/dV kernel left in the scratch (BwdParams::ds): for one 128-query tile of one head, over
// every 128-key tile that sees it, dQ += dS·K with A = dS [128 queries × 128 keys] read M-contiguous from the two
// 64-query dSᵀ tiles (a half the key tile does not see is the scratch's zero tile) and B = K read N-contiguous — one
// tcgen05 product (M 128, N 64, K 128) per key tile, no recomputation of S, P or dP.  Persistent over (query tile,
// head) items, query tiles fastest so consecutive items of a segment reuse its K tiles in L2; a two-stage ring of
// 48 KB stages, two TMEM accumulators so one item's epilogue (dQ rotated back by −θ at the query position, bf16)
// overlaps the next item's MMAs; two CTAs per SM.
//   warp 0      producer: two bulk copies of dSᵀ halves and one TMA load of K per key tile
//   warp 1      TMEM owner and MMA issuer
//   warps 2-5   epilogue, one query row per thread
constexpr int DQG_STAGE = 3 * TILE;
constexpr int DQG_SMEM = 1024 + 2 * DQG_STAGE + 256;
static_assert(2 * DQG_SMEM <= 232448, "two CTAs per SM");

__global__ void __launch_bounds__(192, 2)
    bwd_dq_ds_kernel(const __grid_constant__ CUtensorMap tmk, BwdParams p) {
    constexpr uint32_t IDESC = make_idesc(1, 1, 1, BQ, HD) | (1u << 15) | (1u << 16);   // A (dS), B (K) MN-major
    const int n_tq = *p.n_tq, n_items = n_tq * p.heads;
    if (static_cast<int>(blockIdx.x) >= n_items) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * DQG_STAGE);
    uint64_t* full = bars;            // [2]
    uint64_t* empty = bars + 2;       // [2]
    uint64_t* tfull = bars + 4;       // [2]
    uint64_t* tempty = bars + 6;      // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = warp_id(), lane = lane_id();
    const bool global = p.window < 0;
    const int W = p.window;

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(tfull + b, 1); mbar_init(tempty + b, 4); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 128); tmem_relinquish(); }
    if (warp == 0 && lane == 0) prefetch_tmap(&tmk);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // the key tiles [lo, hi) that see the item's query tile
    struct Item { int head, g, item, q0, L, seg0, first, lo, hi; };
    auto item_of = [&](int it) {
        Item r;
        r.head = it / n_tq;
        r.g = it - r.head * n_tq;
        r.item = p.tq_item[r.g];
        r.q0 = p.tq_p0[r.g];
        r.L = p.seg_len[r.item];
        r.seg0 = p.seg_start[r.item];
        r.first = r.g - r.q0 / BQ;                  // the item's first 128-row tile
        r.lo = global ? 0 : max(0, r.q0 - W) / BK;
        r.hi = global ? (r.L + BK - 1) / BK : (min(r.L, r.q0 + BQ + W) - 1) / BK + 1;
        return r;
    };

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            Item nx = item_of(blockIdx.x);
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const Item m = nx;
                // the next item's geometry is read now, so its latency overlaps this item's loads
                if (it + static_cast<int>(gridDim.x) < n_items) nx = item_of(it + gridDim.x);
                for (int kt = m.lo; kt < m.hi; ++kt, ++g) {
                    const int s = g & 1;
                    if (!mbar_wait(empty + s, ((g >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(full + s, DQG_STAGE);
                    uint8_t* st = smem + s * DQG_STAGE;
                    const int k0 = kt * BK;
                    const int qb0 = global ? 0 : max(0, k0 - W), qe = global ? m.L : min(m.L, k0 + BK + W);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int q = m.q0 + h * BQ2;
                        const size_t idx = (q >= qb0 && q < qe)
                            ? 1 + (static_cast<size_t>(m.first + kt) * p.ds_nq + (q - qb0) / BQ2) * p.heads + m.head : 0;
                        bulk_load(st + h * TILE, p.ds + idx * TILE, TILE, full + s);
                    }
                    tma_load_2d(st + 2 * TILE, &tmk, full + s, p.hidden + m.head * HD, m.seg0 + k0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t g = 0, ti = 0;
            bool ok = true;
            Item nx = item_of(blockIdx.x);
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++ti) {
                const Item m = nx;
                if (it + static_cast<int>(gridDim.x) < n_items) nx = item_of(it + gridDim.x);
                const int buf = ti & 1;
                if (!mbar_wait(tempty + buf, ((ti >> 1) & 1) ^ 1, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(buf * HD);
                for (int kt = m.lo; kt < m.hi; ++kt, ++g) {
                    const int s = g & 1;
                    if (!mbar_wait(full + s, (g >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = smem_u32(smem + s * DQG_STAGE), b = a + 2 * TILE;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_f16(d, desc_mn_sw128(a + kk * 2048, TILE), desc_mn_sw128(b + kk * 2048, TILE), IDESC,
                                (kt > m.lo || kk > 0) ? 1u : 0u);
                    mma_commit(empty + s);
                }
                mma_commit(tfull + buf);
            }
        }
    } else {
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        uint32_t ti = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++ti) {
            const Item m = item_of(it);
            const int buf = ti & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(tfull + buf, (ti >> 1) & 1, abort_flag, p.err))) break;
            tc_fence_after();
            uint32_t x[32], y[32];
            tmem_ld32(tmem + lane_off + static_cast<uint32_t>(buf * HD), x);
            tmem_ld32(tmem + lane_off + static_cast<uint32_t>(buf * HD + 32), y);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty + buf);
            const int q = m.q0 + row;
            if (q < m.L) {
                float a[32], b[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) { a[e] = __uint_as_float(x[e]); b[e] = __uint_as_float(y[e]); }
                if (p.cosv) {   // pairs (i, i + 32) rotated back by −θ at the query's position (16-byte aligned tables)
                    const float4* c4 = reinterpret_cast<const float4*>(p.cosv + static_cast<size_t>(q) * (HD / 2));
                    const float4* s4 = reinterpret_cast<const float4*>(p.sinv + static_cast<size_t>(q) * (HD / 2));
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const float4 c = __ldg(c4 + t), sn = __ldg(s4 + t);
                        const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
                        for (int u4 = 0; u4 < 4; ++u4) {
                            const int i = 4 * t + u4;
                            const float u = a[i], v = b[i];
                            a[i] = __fadd_rn(__fmul_rn(u, cc[u4]), __fmul_rn(v, ss[u4]));
                            b[i] = __fsub_rn(__fmul_rn(v, cc[u4]), __fmul_rn(u, ss[u4]));
                        }
                    }
                }
                __nv_bfloat16* out = p.dqkv + static_cast<size_t>(m.seg0 + q) * p.lddq + m.head * HD;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    *reinterpret_cast<uint4*>(out + 8 * t) =
                        make_uint4(pack2(a[8 * t], a[8 * t + 1]), pack2(a[8 * t + 2], a[8 * t + 3]),
                                   pack2(a[8 * t + 4], a[8 * t + 5]), pack2(a[8 * t + 6], a[8 * t + 7]));
                    *reinterpret_cast<uint4*>(out + 32 + 8 * t) =
                        make_uint4(pack2(b[8 * t], b[8 * t + 1]), pack2(b[8 * t + 2], b[8 * t + 3]),
                                   pack2(b[8 * t + 4], b[8 * t + 5]), pack2(b[8 * t + 6], b[8 * t + 7]));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
}

}  // namespace fat

template <bool SPLIT, bool DROP>
static int launch_tc(const fa::Args& a, cudaStream_t s) {
    using C = fat::Cfg<SPLIT>;
    CUtensorMap th, tl;
    int rc = make_tmap_2d(&th, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                          static_cast<uint64_t>(a.ld) * 2, fat::BK, fat::HD, true);
    if (!rc) rc = make_tmap_2d(&tl, SPLIT ? a.qkv_lo : a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                               static_cast<uint64_t>(a.ld) * 2, fat::BK, fat::HD, true);
    if (rc) return rc;
    static DeviceOnce attr;
    int dev = 0, nsm = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(fat::fwd_tc_kernel<SPLIT, DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM));
        attr.mark(dev);
    }
    if (int e = sm_count(dev, &nsm)) return e;
    fat::Params p{};
    p.seg_start = a.seg_start; p.seg_len = a.seg_len;
    p.tq_item = a.tq_item; p.tq_p0 = a.tq_p0; p.n_tq = a.n_tq;
    p.window = a.window; p.hidden = a.hidden; p.heads = a.heads;
    p.scale = a.scale; p.dropout = a.dropout; p.keep = a.keep; p.seed = a.seed;
    p.out = a.out; p.out_lo = a.out_lo; p.ldo = a.ldo; p.lse = a.lse; p.err = a.err;
    const int items = a.max_tq * a.heads;
    fat::fwd_tc_kernel<SPLIT, DROP><<<items < nsm ? items : nsm, 320, C::SMEM, s>>>(th, tl, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

// The decision forward's attention on the tensor cores (head_dim 64): q, k, v already rotated, fp16 [T, ld], the
// context out as Q8_0 codes and scales.
template <int MODE>
static int launch_infer_tc(const InferAttn& a, cudaStream_t s) {
    using C = fat::Cfg<false>;
    CUtensorMap th;
    int rc = make_tmap_2d(&th, a.qkv16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.T, 3 * a.hidden,
                          static_cast<uint64_t>(a.ld) * 2, fat::BK, fat::HD, true);
    if (rc) return rc;
    static DeviceOnce attr;
    int dev = 0, nsm = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(fat::fwd_tc_kernel<false, false, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM));
        attr.mark(dev);
    }
    if (int e = sm_count(dev, &nsm)) return e;
    fat::Params p{};
    p.seg_start = a.seg_start; p.seg_len = a.seg_len;
    p.tq_item = a.tq_item; p.tq_p0 = a.tq_p0; p.n_tq = a.n_tq;
    p.window = a.window; p.hidden = a.hidden; p.heads = a.heads;
    p.scale = a.scale; p.keep = 1.0f;
    p.q8 = a.q; p.q8d = a.d; p.q8ldd = a.ldd; p.err = a.err;
    p.out = a.hi; p.out_lo = a.lo; p.ldo = a.hidden;
    const int items = a.max_tq * a.heads;
    fat::fwd_tc_kernel<false, false, MODE><<<items < nsm ? items : nsm, 320, C::SMEM, s>>>(th, th, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int flash_forward_tc_q8(const InferAttn& a, cudaStream_t s) {
    if (a.hidden / a.heads != fat::HD || a.max_tq <= 0 || a.T <= 0) return ERR_NOT_SUPPORTED;
    if ((a.ld & 7) || (reinterpret_cast<uintptr_t>(a.qkv16) & 15)) return ERR_NOT_SUPPORTED;
    if (a.q) return launch_infer_tc<1>(a, s);
    if (!a.hi || !a.lo || (reinterpret_cast<uintptr_t>(a.hi) & 15) || (reinterpret_cast<uintptr_t>(a.lo) & 15))
        return ERR_NOT_SUPPORTED;
    return launch_infer_tc<2>(a, s);
}

// The tcgen05 forward for head_dim 64; returns ERR_NOT_SUPPORTED for shapes it does not take (the caller then runs
// the mma.sync forward).
int flash_forward_tc(const fa::Args& a, cudaStream_t s) {
    if (a.hidden / a.heads != fat::HD || !a.tq_item || a.max_tq <= 0 || a.T <= 0) return ERR_NOT_SUPPORTED;
    if ((a.ld & 7) || (reinterpret_cast<uintptr_t>(a.qkv) & 15) || (a.qkv_lo && (reinterpret_cast<uintptr_t>(a.qkv_lo) & 15)))
        return ERR_NOT_SUPPORTED;
    if (a.qkv_lo && !a.out_lo) { set_error("accurate attention needs the context's low part"); return ERR_ARGUMENT; }
    const bool drop = a.dropout > 0.f;
    if (a.qkv_lo) return drop ? launch_tc<true, true>(a, s) : launch_tc<true, false>(a, s);
    return drop ? launch_tc<false, true>(a, s) : launch_tc<false, false>(a, s);
}

template <bool DROP>
static int launch_bwd_tc(const fa::Args& a, cudaStream_t s) {
    CUtensorMap tk, tq, tdo;
    int rc = make_tmap_2d(&tk, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                          static_cast<uint64_t>(a.ld) * 2, fat::BK, fat::HD, true);
    if (!rc) rc = make_tmap_2d(&tq, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                               static_cast<uint64_t>(a.ld) * 2, fat::BQ2, fat::HD, true);
    if (!rc) rc = make_tmap_2d(&tdo, a.dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, a.hidden,
                               static_cast<uint64_t>(a.ldo) * 2, fat::BQ2, fat::HD, true);
    if (rc) return rc;
    static DeviceOnce attr;
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(fat::bwd_dkdv_tc_kernel<DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       fat::BWD_SMEM));
        attr.mark(dev);
    }
    fat::BwdParams p{};
    p.seg_start = a.seg_start; p.seg_len = a.seg_len;
    p.tq_item = a.tq_item; p.tq_p0 = a.tq_p0; p.n_tq = a.n_tq;
    p.window = a.window; p.hidden = a.hidden; p.heads = a.heads;
    p.scale = a.scale; p.dropout = a.dropout; p.keep = a.keep; p.seed = a.seed;
    p.lse = a.lse; p.dsum = a.dsum; p.cosv = a.cosv; p.sinv = a.sinv;
    p.dqkv = a.dqkv; p.lddq = a.lddq; p.err = a.err;
    p.ds = a.ds; p.ds_nq = a.ds_nq;
    p.dmask = a.dmask; p.dmask_w = a.dmask_w; p.dmask_rows = a.dmask_rows;
    int nsm = 0;
    if (int e = sm_count(dev, &nsm)) return e;
    p.wave = 2 * nsm;
    fat::bwd_dkdv_tc_kernel<DROP><<<dim3(a.max_tq, a.heads), 320, fat::BWD_SMEM, s>>>(tk, tq, tdo, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

// dK and dV by the tcgen05 kernel for head_dim 64 (ERR_NOT_SUPPORTED for shapes it does not take).
int flash_backward_dkdv_tc(const fa::Args& a, cudaStream_t s) {
    if (a.hidden / a.heads != fat::HD || !a.tq_item || a.max_tq <= 0 || a.T <= 0) return ERR_NOT_SUPPORTED;
    if ((a.ld & 7) || (a.ldo & 7) || (a.lddq & 7) || (reinterpret_cast<uintptr_t>(a.qkv) & 15) ||
        (reinterpret_cast<uintptr_t>(a.dout) & 15) || (reinterpret_cast<uintptr_t>(a.dqkv) & 15) ||
        (reinterpret_cast<uintptr_t>(a.cosv) & 15) || (reinterpret_cast<uintptr_t>(a.sinv) & 15))
        return ERR_NOT_SUPPORTED;
    return a.dropout > 0.f ? launch_bwd_tc<true>(a, s) : launch_bwd_tc<false>(a, s);
}

template <bool DROP>
static int launch_dq_tc(const fa::Args& a, cudaStream_t s) {
    CUtensorMap tq, tkv, tdo;
    int rc = make_tmap_2d(&tq, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                          static_cast<uint64_t>(a.ld) * 2, fat::BQ, fat::HD, true);
    if (!rc) rc = make_tmap_2d(&tkv, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                               static_cast<uint64_t>(a.ld) * 2, fat::DQ_BK, fat::HD, true);
    if (!rc) rc = make_tmap_2d(&tdo, a.dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, a.hidden,
                               static_cast<uint64_t>(a.ldo) * 2, fat::BQ, fat::HD, true);
    if (rc) return rc;
    static DeviceOnce attr;
    int dev = 0, nsm = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(fat::bwd_dq_tc_kernel<DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       fat::DQ_SMEM));
        attr.mark(dev);
    }
    if (int e = sm_count(dev, &nsm)) return e;
    fat::BwdParams p{};
    p.seg_start = a.seg_start; p.seg_len = a.seg_len;
    p.tq_item = a.tq_item; p.tq_p0 = a.tq_p0; p.n_tq = a.n_tq;
    p.window = a.window; p.hidden = a.hidden; p.heads = a.heads;
    p.scale = a.scale; p.dropout = a.dropout; p.keep = a.keep; p.seed = a.seed;
    p.lse = a.lse; p.dsum = a.dsum; p.cosv = a.cosv; p.sinv = a.sinv;
    p.dqkv = a.dqkv; p.lddq = a.lddq; p.err = a.err;
    p.ds = nullptr; p.ds_nq = 0;
    const int items = a.max_tq * a.heads, slots = 2 * nsm;   // 2 CTAs per SM
    fat::bwd_dq_tc_kernel<DROP><<<items < slots ? items : slots, 320, fat::DQ_SMEM, s>>>(tq, tkv, tdo, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

// dQ = dS·K from the scratch the dK/dV kernel filled (run after it); ERR_NOT_SUPPORTED without a scratch or for
// shapes it does not take.
int flash_backward_dq_ds(const fa::Args& a, cudaStream_t s) {
    if (!a.ds || a.ds_nq <= 0 || a.hidden / a.heads != fat::HD || !a.tq_item || a.max_tq <= 0 || a.T <= 0)
        return ERR_NOT_SUPPORTED;
    if ((a.window >= 0 && a.window % fat::BQ2) || (a.ld & 7) || (a.lddq & 7) ||
        (reinterpret_cast<uintptr_t>(a.qkv) & 15) || (reinterpret_cast<uintptr_t>(a.dqkv) & 15) ||
        (reinterpret_cast<uintptr_t>(a.ds) & 15) || (reinterpret_cast<uintptr_t>(a.cosv) & 15) ||
        (reinterpret_cast<uintptr_t>(a.sinv) & 15))
        return ERR_NOT_SUPPORTED;
    CUtensorMap tk;
    if (int rc = make_tmap_2d(&tk, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.T, 3 * a.hidden,
                              static_cast<uint64_t>(a.ld) * 2, fat::BK, fat::HD, true))
        return rc;
    static DeviceOnce attr;
    int dev = 0, nsm = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(fat::bwd_dq_ds_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fat::DQG_SMEM));
        attr.mark(dev);
    }
    if (int e = sm_count(dev, &nsm)) return e;
    fat::BwdParams p{};
    p.seg_start = a.seg_start; p.seg_len = a.seg_len;
    p.tq_item = a.tq_item; p.tq_p0 = a.tq_p0; p.n_tq = a.n_tq;
    p.window = a.window; p.hidden = a.hidden; p.heads = a.heads;
    p.cosv = a.cosv; p.sinv = a.sinv;
    p.dqkv = a.dqkv; p.lddq = a.lddq; p.err = a.err;
    p.ds = a.ds; p.ds_nq = a.ds_nq;
    const int items = a.max_tq * a.heads, slots = 2 * nsm;
    fat::bwd_dq_ds_kernel<<<items < slots ? items : slots, 192, fat::DQG_SMEM, s>>>(tk, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

// dQ by the tcgen05 kernel for head_dim 64 (ERR_NOT_SUPPORTED for shapes it does not take).
int flash_backward_dq_tc(const fa::Args& a, cudaStream_t s) {
    if (a.hidden / a.heads != fat::HD || !a.tq_item || a.max_tq <= 0 || a.T <= 0) return ERR_NOT_SUPPORTED;
    if ((a.ld & 7) || (a.ldo & 7) || (a.lddq & 7) || (reinterpret_cast<uintptr_t>(a.qkv) & 15) ||
        (reinterpret_cast<uintptr_t>(a.dout) & 15) || (reinterpret_cast<uintptr_t>(a.dqkv) & 15))
        return ERR_NOT_SUPPORTED;
    return a.dropout > 0.f ? launch_dq_tc<true>(a, s) : launch_dq_tc<false>(a, s);
}

}  // namespace laya
