// gemm_bf16.cu — the bf16 tensor-core products of the training step (sm_100a tcgen05, fp32 accumulation in TMEM).
//
// Replaces the fp32 panel GEMM of the reference's training path (PackedMatrix.Multiply, Base/Numerics/PackedMatrix.cs:
// 121-305) as used by Ops.Linear / Ops.LinearBackward (Laya.Training/Ops.cs:22-69):
//     forward   y  = x · Wᵀ (+ b)          A = x  [T, K] K-major,        B = W  [N, K] K-major
//     input     dx = dy · W                 A = dy [T, N] K-major,        B = W  [N, K] read MN-major (K contiguous)
//     weight    dW += dyᵀ · x               A = dy [T, N] read MN-major,  B = x  [T, K] read MN-major
// Operand majorness is a bit of the tcgen05 instruction descriptor plus the shared-memory descriptor layout, so no
// operand is ever transposed in memory (the reference transposes dy and repacks x for every dW, Ops.cs:43-62).
//
// CTA layout: persistent, one CTA per SM, tiles of 128 × BN walked N-fastest.
//   warp 0      TMA producer, STAGES-deep ring of A and B tiles (64 codes of K per stage = one 128-byte swizzle row).
//   warp 1      TMEM allocator and MMA issuer: 4 × (M=128, N=BN, K=16) per stage into one of two TMEM accumulators,
//               so the epilogue of one tile overlaps the MMAs of the next.
//   warps 2-9   epilogue: 4 lane quarters × 2 column halves; each drains 32-column chunks with tcgen05.ld, adds the
//               bias, converts, stages 32 rows × 128 B in shared memory and writes them with one TMA store (or TMA
//               reduce-add for accumulating outputs: residual streams and parameter gradients).
#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "ksplit.h"
#include "train.h"

namespace laya {
namespace bf {

constexpr int BM = 128;
constexpr int BK = 64;           // bf16 per 128-byte row
constexpr int EPI_WARPS = 8;

template <int BN, int STAGES>
struct Cfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGE_OUT = 4096;
    static constexpr int THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int BAR_BYTES = 8 * (2 * STAGES + 4) + 16;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_WARPS * STAGE_OUT + BAR_BYTES;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(2 * BN <= 512, "two TMEM accumulators");
};

// MN-major operand, 128-byte swizzle: 64-element MN atoms of BK rows each (LBO apart), 8-row K groups 1024 B apart.
DEVI uint64_t smem_desc_mn_sw128(uint32_t saddr, uint32_t lbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

struct KParams {
    int M, N, K;
    int splits;        // 1: A·Bᵀ;  2: A·Bᵀ + A2·Bᵀ (B exactly bf16);  3: A·Bᵀ + A2·Bᵀ + A·B2ᵀ (hi/lo operand
                       // pairs, an fp32-accurate product)
    int ksplit;        // K chunks per output tile (accumulating outputs only: chunks reduce-add into the output)
    const float* bias;
    int* err;
    // EPI_QKV: rotary tables [position, 32] (null: no rotation), each row's position, the rotated columns
    const int32_t* tok_item; const int32_t* seg_start; const float* cosv; const float* sinv; int rot_cols;
};

// Drains one warp's share of an accumulator — 32 TMEM lanes (rows gr0..gr0+31) × cols columns from gc0, cols a
// multiple of 64 — adds the bias, converts, and writes it through a 4 KB staging tile with TMA stores (reduce-adds for
// EPI_F32_ADD).
template <int EPI>
DEVI void drain_rows(uint32_t tbase, uint8_t* stage, const CUtensorMap* tmOut, const float* bias, int N, int gc0,
                     int gr0, int lane, int cols) {
    if constexpr (EPI == EPI_BF16) {
        // 64 columns per chunk: 64 bf16 = one 128-byte swizzled row per lane
#pragma unroll 1
        for (int c = 0; c < cols / 64; ++c) {
            uint32_t v0[32], v1[32];
            tmem_ld32(tbase + c * 64, v0);
            tmem_ld32(tbase + c * 64 + 32, v1);
            tmem_ld_wait();
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                uint32_t w[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int j = q * 8 + 2 * t;
                    float lo = __uint_as_float(j < 32 ? v0[j] : v1[j - 32]);
                    float hi = __uint_as_float(j + 1 < 32 ? v0[j + 1] : v1[j + 1 - 32]);
                    if (bias) {
                        const int col = gc0 + c * 64 + j;
                        lo += col < N ? __ldg(bias + col) : 0.0f;
                        hi += col + 1 < N ? __ldg(bias + col + 1) : 0.0f;
                    }
                    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
                    w[t] = *reinterpret_cast<uint32_t*>(&h);
                }
                *reinterpret_cast<uint4*>(stage + lane * 128 + ((q ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) { tma_store_2d(tmOut, gc0 + c * 64, gr0, stage); bulk_commit(); }
        }
    } else {
#pragma unroll 1
        for (int c = 0; c < cols / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(tbase + c * 32, v);
            tmem_ld_wait();
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 f;
                float* fp = &f.x;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int j = q * 4 + t;
                    float x = __uint_as_float(v[j]);
                    if (bias) {
                        const int col = gc0 + c * 32 + j;
                        x += col < N ? __ldg(bias + col) : 0.0f;
                    }
                    fp[t] = x;
                }
                *reinterpret_cast<float4*>(stage + lane * 128 + ((q ^ (lane & 7)) << 4)) = f;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if constexpr (EPI == EPI_F32_ADD) tma_reduce_add_2d(tmOut, gc0 + c * 32, gr0, stage);
                else tma_store_2d(tmOut, gc0 + c * 32, gr0, stage);
                bulk_commit();
            }
        }
    }
}

// The attention input's epilogue (EPI_QKV): 64-column chunks, each one head of q, k or v (chunks start on multiples of
// 64 and the q | k | v boundaries are multiples of 64), so a thread holds both halves (i, i + 32) of its row's
// rotation pairs: columns below rot_cols are rotated at the row's segment position in the reference's fp32 order
// (Rotary.Apply, Ops.cs:490-503: x·c − y·s, y·c + x·s), then written as bf16 hi through tmOut and, with has_lo, the
// bf16 remainder x − bf16(x) through tmOut2.
// The row's position for the rotation (−1: the row is not rotated), found before the caller waits for the accumulator
// and with the row's two 128-byte table lines (32 cosines, 32 sines) prefetched into L1, so these dependent loads
// overlap the wait.
DEVI int qkv_rot_pos(const KParams& p, int row, int gc0) {
    if (!p.cosv || row >= p.M || gc0 >= p.rot_cols) return -1;
    const int pos = row - p.seg_start[p.tok_item[row]];
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p.cosv + static_cast<size_t>(pos) * 32));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p.sinv + static_cast<size_t>(pos) * 32));
    return pos;
}
DEVI void drain_qkv(uint32_t tbase, uint8_t* stage, const CUtensorMap* tmOut, const CUtensorMap* tmOut2, bool has_lo,
                    const KParams& p, const float* bias, int gc0, int gr0, int lane, int cols, int pos) {
#pragma unroll 1
    for (int c = 0; c < cols / 64; ++c) {
        uint32_t v0[32], v1[32];
        tmem_ld32(tbase + c * 64, v0);
        tmem_ld32(tbase + c * 64 + 32, v1);
        tmem_ld_wait();
        const int col0 = gc0 + c * 64;
        float x[64];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            x[j] = __uint_as_float(v0[j]);
            x[32 + j] = __uint_as_float(v1[j]);
        }
        if (bias) {
#pragma unroll
            for (int j = 0; j < 64; ++j) x[j] += col0 + j < p.N ? __ldg(bias + col0 + j) : 0.0f;
        }
        if (pos >= 0 && col0 < p.rot_cols) {   // 16-byte aligned tables (checked at launch): four-wide loads
            const float4* c4 = reinterpret_cast<const float4*>(p.cosv + static_cast<size_t>(pos) * 32);
            const float4* s4 = reinterpret_cast<const float4*>(p.sinv + static_cast<size_t>(pos) * 32);
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const float4 c = __ldg(c4 + t), sv = __ldg(s4 + t);
                const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                for (int u4 = 0; u4 < 4; ++u4) {
                    const int j = 4 * t + u4;
                    const float u = x[j], v = x[32 + j];
                    x[j] = __fsub_rn(__fmul_rn(u, cc[u4]), __fmul_rn(v, ss[u4]));
                    x[32 + j] = __fadd_rn(__fmul_rn(v, cc[u4]), __fmul_rn(u, ss[u4]));
                }
            }
        }
#pragma unroll 1
        for (int part = 0; part < (has_lo ? 2 : 1); ++part) {
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                uint32_t w[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float a = x[q * 8 + 2 * t], b = x[q * 8 + 2 * t + 1];
                    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
                    if (part == 1)
                        h = __floats2bfloat162_rn(a - __bfloat162float(h.x), b - __bfloat162float(h.y));
                    w[t] = *reinterpret_cast<uint32_t*>(&h);
                }
                *reinterpret_cast<uint4*>(stage + lane * 128 + ((q ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) { tma_store_2d(part ? tmOut2 : tmOut, col0, gr0, stage); bulk_commit(); }
        }
    }
}

template <int BN, int STAGES, int A_MN, int B_MN, int EPI>
__global__ void __launch_bounds__(Cfg<BN, STAGES>::THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                     const __grid_constant__ CUtensorMap tmOut, KParams p) {
    using C = Cfg<BN, STAGES>;
    constexpr uint32_t IDESC = make_idesc(/*D f32*/ 1, /*A bf16*/ 1, /*B bf16*/ 1, BM, BN) |
                               (static_cast<uint32_t>(A_MN) << 15) | (static_cast<uint32_t>(B_MN) << 16);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint8_t* sOut = smem + STAGES * C::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sOut + EPI_WARPS * C::STAGE_OUT);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = warp_id(), lane = lane_id();
    const int kblocks = (p.K + BK - 1) / BK;
    const int kchunk = (kblocks + p.ksplit - 1) / p.ksplit;   // k-blocks per work unit
    const int tiles_n = (p.N + BN - 1) / BN;
    const int tiles = tiles_n * ((p.M + BM - 1) / BM) * p.ksplit;   // work units: (output tile, K chunk)
    // unit u: output tile u / ksplit, k-blocks [kb0, kb0 + nkb); split passes (A, B), (A2, B), (A, B2) per k-block
    auto unit_k = [&](int u, int& kb0, int& nkb) {
        kb0 = (u % p.ksplit) * kchunk;
        nkb = min(kchunk, kblocks - kb0);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(tfull + b, 1); mbar_init(tempty + b, EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA); prefetch_tmap(&tmB); prefetch_tmap(&tmOut);
        if (p.splits > 1) { prefetch_tmap(&tmA2); prefetch_tmap(&tmB2); }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int ot = tile / p.ksplit;
                const int m0 = (ot / tiles_n) * BM, n0 = (ot % tiles_n) * BN;
                int kb0, nkb;
                unit_k(tile, kb0, nkb);
                const int iters = nkb * p.splits;
                for (int it = 0; it < iters; ++it, ++g) {
                    const int s = g % STAGES;
                    const int seg = it / nkb, kb = kb0 + it - seg * nkb;
                    const CUtensorMap* mA = seg == 1 ? &tmA2 : &tmA;
                    const CUtensorMap* mB = seg == 2 ? &tmB2 : &tmB;
                    if (!mbar_wait(empty + s, ((g / STAGES) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(full + s, C::STAGE_BYTES);
                    uint8_t* a = sA + s * C::A_BYTES;
                    uint8_t* b = sB + s * C::B_BYTES;
                    if constexpr (A_MN) {
#pragma unroll
                        for (int j = 0; j < BM / 64; ++j) tma_load_2d(a + j * (BK * 128), mA, full + s, m0 + 64 * j, kb * BK);
                    } else {
                        tma_load_2d(a, mA, full + s, kb * BK, m0);
                    }
                    if constexpr (B_MN) {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * (BK * 128), mB, full + s, n0 + 64 * j, kb * BK);
                    } else {
                        tma_load_2d(b, mB, full + s, kb * BK, n0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t g = 0, ti = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++ti) {
                const int buf = ti & 1;
                if (!mbar_wait(tempty + buf, ((ti >> 1) & 1) ^ 1, abort_flag, p.err)) break;
                tc_fence_after();
                int kb0, nkb;
                unit_k(tile, kb0, nkb);
                const int iters = nkb * p.splits;
                for (int kb = 0; kb < iters; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (!mbar_wait(full + s, (g / STAGES) & 1, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = smem_u32(sA + s * C::A_BYTES), b = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad = A_MN ? smem_desc_mn_sw128(a + kk * 2048, BK * 128) : smem_desc_sw128(a + kk * 32);
                        const uint64_t bd = B_MN ? smem_desc_mn_sw128(b + kk * 2048, BK * 128) : smem_desc_sw128(b + kk * 32);
                        mma_f16(tmem + static_cast<uint32_t>(buf * BN), ad, bd, IDESC, (kb | kk) != 0 ? 1u : 0u);
                    }
                    mma_commit(empty + s);
                }
                mma_commit(tfull + buf);
            }
        }
    } else {
        const int e = warp - 2;
        const int quarter = warp & 3;
        const int half = e >> 2;
        constexpr int COLS = BN / 2;
        uint8_t* stage = sOut + e * C::STAGE_OUT;
        uint32_t ti = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++ti) {
            const int buf = ti & 1;
            const int ot = tile / p.ksplit;
            const int m0 = (ot / tiles_n) * BM, n0 = (ot % tiles_n) * BN;
            const float* bias = tile % p.ksplit == 0 ? p.bias : nullptr;   // once per output tile
            if (!mbar_wait(tfull + buf, (ti >> 1) & 1, abort_flag, p.err)) break;
            tc_fence_after();
            const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN + half * COLS);
            const int gc0 = n0 + half * COLS;
            const int gr0 = m0 + quarter * 32;
            drain_rows<EPI>(tbase, stage, &tmOut, bias, p.N, gc0, gr0, lane, COLS);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty + buf);
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------------ CTA-pair form
// Output tiles of 256 × 256 over a cluster of two CTAs (the SM pair of one TPC). Each CTA loads its own 128 rows of
// A and its own 128 rows of B's N per stage — 32 KB instead of the 48 KB a one-CTA 128 × 256 tile loads for the same
// MMA work, so shared-memory fill and L2 → SM traffic per flop drop by a third — and the even rank issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256) reading both CTAs' stages. Each CTA's TMEM holds its 128 rows of the
// accumulator (two buffers of 256 columns) and its own epilogue warps drain them exactly as in the one-CTA kernel.
//   full[s]   even rank only: its producer arms it with both CTAs' bytes; both CTAs' loads complete on it.
//   empty[s]  in both CTAs: the MMA issuer commits to its own and to the peer's when a stage is consumed.
//   tfull[b]  in both CTAs: committed likewise when an accumulator buffer is complete.
//   tempty[b] even rank only: all 16 epilogue warps of the pair arrive when a buffer is drained.
// No load is multicast; the pair exchanges only mbarrier arrivals and the MMA's own operand traffic.
//
// Narrow units (256 × 128, N = 128 per MMA, 64 B rows per CTA): the last tile column when N mod 256 is in (0, 128],
// so no MMA work is spent past N, and every tile of a last partial round of tiles when that round holds at most half
// the pairs — split in two along N, it ends in half the time (240 tiles of N = 768 on 74 pairs: 3 full rounds and 18
// tiles, which become 36 narrow units).
constexpr int PAIR_BN = 256;

// SPL: the operand parts one stage carries for a k-block — 1: A, B; 2: A, A2, B (A·Bᵀ + A2·Bᵀ); 3: A, A2, B, B2
// (A·Bᵀ + A2·Bᵀ + A·B2ᵀ, the hi/lo passes of an fp32-accurate product).  Each part is loaded once per k-block and the
// stage's MMAs take every pass from it, so a split product moves 4 tiles per k-block instead of 6.
template <int STAGES, int SPL>
struct PairCfg {
    static constexpr int A_BYTES = BM * BK * 2;                  // this CTA's 128 rows of A
    static constexpr int B_BYTES = (PAIR_BN / 2) * BK * 2;       // this CTA's 128 rows of B (64 for a narrow unit)
    static constexpr int NA = SPL >= 2 ? 2 : 1;                  // A parts per stage (hi, lo)
    static constexpr int NB = SPL == 3 ? 2 : 1;                  // B parts per stage
    static constexpr int STAGE_BYTES = NA * A_BYTES + NB * B_BYTES;
    static constexpr int STAGE_OUT = 4096;
    static constexpr int THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int BAR_BYTES = 8 * (2 * STAGES + 4) + 16;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_WARPS * STAGE_OUT + BAR_BYTES;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct PairParams {
    KParams k;
    int units;        // work units walked by the pairs
    int split_from;   // units from here on are the halves of tiles split along N (split_from + 2·(tiles − split_from))
    int has_lo;       // EPI_QKV: the low parts are written too
};

// One work unit of the pair kernel: output rows [m0, m0 + 256), columns [n0, n0 + (wide ? 256 : 128)), k-blocks
// [kb0, kb0 + nkb); skip for the empty second half of a tile that was narrow already.
struct PairUnit {
    int m0, n0, kb0, nkb;
    bool wide, first, skip;
};

DEVI PairUnit pair_unit(const PairParams& pp, int u, int tiles_n, int kchunk, int kblocks) {
    const KParams& p = pp.k;
    int tile = u, half = -1;
    if (u >= pp.split_from) {
        tile = pp.split_from + ((u - pp.split_from) >> 1);
        half = (u - pp.split_from) & 1;
    }
    const int ot = tile / p.ksplit;
    const int nt = ot % tiles_n;
    PairUnit r;
    r.m0 = (ot / tiles_n) * (2 * BM);
    r.n0 = nt * PAIR_BN;
    r.wide = !(nt == tiles_n - 1 && p.N - r.n0 <= PAIR_BN / 2);
    r.skip = false;
    if (half >= 0) {
        if (r.wide) { r.n0 += (PAIR_BN / 2) * half; r.wide = false; }
        else r.skip = half == 1;
    }
    r.kb0 = (tile % p.ksplit) * kchunk;
    r.nkb = min(kchunk, kblocks - r.kb0);
    r.first = tile % p.ksplit == 0;
    return r;
}

template <int STAGES, int SPL, int A_MN, int B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<STAGES, SPL>::THREADS, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                          const __grid_constant__ CUtensorMap tmBn, const __grid_constant__ CUtensorMap tmB2n,
                          const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmOut2,
                          PairParams pp) {
    using C = PairCfg<STAGES, SPL>;
    constexpr int BN = PAIR_BN;
    constexpr uint32_t IDESC_BASE = (static_cast<uint32_t>(A_MN) << 15) | (static_cast<uint32_t>(B_MN) << 16);
    constexpr uint32_t IDESC_WIDE = make_idesc(/*D f32*/ 1, /*A bf16*/ 1, /*B bf16*/ 1, 2 * BM, BN) | IDESC_BASE;
    constexpr uint32_t IDESC_NARROW = make_idesc(1, 1, 1, 2 * BM, BN / 2) | IDESC_BASE;
    const KParams& p = pp.k;
    extern __shared__ uint8_t smem_raw[];
    // both CTAs run the same code on the same dynamic-shared-memory base, so every buffer sits at the same offset in
    // both: the MMA's descriptors and the mapa'd barrier addresses rely on it
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // stage s: [A | A2 | B | B2] (the parts SPL carries), each 1024-aligned
    auto part_a = [&](int s, int i) { return smem + s * C::STAGE_BYTES + i * C::A_BYTES; };
    auto part_b = [&](int s, int i) { return smem + s * C::STAGE_BYTES + C::NA * C::A_BYTES + i * C::B_BYTES; };
    uint8_t* sOut = smem + STAGES * C::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sOut + EPI_WARPS * C::STAGE_OUT);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = warp_id(), lane = lane_id();
    const uint32_t rank = cluster_rank();          // 0: issues the MMAs; 1: its peer
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int kblocks = (p.K + BK - 1) / BK;
    const int kchunk = (kblocks + p.ksplit - 1) / p.ksplit;
    const int tiles_n = (p.N + BN - 1) / BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(tfull + b, 1); mbar_init(tempty + b, 2 * EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc_pair(tmem_slot, 512); tmem_relinquish_pair(); }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA); prefetch_tmap(&tmB); prefetch_tmap(&tmOut);
        if (p.splits > 1) { prefetch_tmap(&tmA2); prefetch_tmap(&tmB2); }
    }
    // barriers initialised in both CTAs before either side arrives on, or loads into, the other's
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full0 = cluster_addr(full, 0);    // the even rank's full barriers
            uint32_t g = 0;
            bool ok = true;
            for (int u = pair; u < pp.units && ok; u += npairs) {
                const PairUnit w = pair_unit(pp, u, tiles_n, kchunk, kblocks);
                if (w.skip) continue;
                const int bn = w.wide ? BN / 2 : BN / 4;     // B rows (N) this CTA loads
                const int m0 = w.m0 + static_cast<int>(rank) * BM;
                const int n0 = w.n0 + static_cast<int>(rank) * bn;
                const uint32_t bytes = 2u * static_cast<uint32_t>(C::NA * C::A_BYTES + C::NB * bn * BK * 2);
                for (int it = 0; it < w.nkb; ++it, ++g) {
                    const int s = g % STAGES;
                    const int kb = w.kb0 + it;
                    if (!mbar_wait(empty + s, ((g / STAGES) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    if (rank == 0) mbar_arrive_expect_tx(full + s, bytes);
                    const uint32_t bar = full0 + 8u * static_cast<uint32_t>(s);
#pragma unroll
                    for (int i = 0; i < C::NA; ++i) {
                        const CUtensorMap* mA = i ? &tmA2 : &tmA;
                        uint8_t* a = part_a(s, i);
                        if constexpr (A_MN) {
#pragma unroll
                            for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(a + j * (BK * 128), mA, bar, m0 + 64 * j, kb * BK);
                        } else {
                            tma_load_2d_pair(a, mA, bar, kb * BK, m0);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < C::NB; ++i) {
                        const CUtensorMap* mB = i ? (w.wide || B_MN ? &tmB2 : &tmB2n) : (w.wide || B_MN ? &tmB : &tmBn);
                        uint8_t* b = part_b(s, i);
                        if constexpr (B_MN) {
                            for (int j = 0; j < bn / 64; ++j) tma_load_2d_pair(b + j * (BK * 128), mB, bar, n0 + 64 * j, kb * BK);
                        } else {
                            tma_load_2d_pair(b, mB, bar, kb * BK, n0);
                        }
                    }
                }
            }
            // every stage's last use released before this CTA may exit (the issuer's commits land in this CTA)
            for (int i = 0; i < STAGES && ok; ++i, ++g)
                if (!mbar_wait(empty + g % STAGES, ((g / STAGES) & 1) ^ 1, abort_flag, p.err)) ok = false;
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            const uint32_t empty1 = cluster_addr(empty, 1), tfull1 = cluster_addr(tfull, 1);
            uint32_t g = 0, ti = 0;
            bool ok = true;
            for (int u = pair; u < pp.units && ok; u += npairs) {
                const PairUnit w = pair_unit(pp, u, tiles_n, kchunk, kblocks);
                if (w.skip) continue;
                const uint32_t idesc = w.wide ? IDESC_WIDE : IDESC_NARROW;
                const int buf = ti & 1;
                if (!mbar_wait(tempty + buf, ((ti >> 1) & 1) ^ 1, abort_flag, p.err)) break;
                tc_fence_after();
                for (int kb = 0; kb < w.nkb; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (!mbar_wait(full + s, (g / STAGES) & 1, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(part_a(s, 0)), a1 = smem_u32(part_a(s, C::NA - 1));
                    const uint32_t b0 = smem_u32(part_b(s, 0)), b1 = smem_u32(part_b(s, C::NB - 1));
                    auto desc_a = [&](uint32_t a, int kk) {
                        return A_MN ? smem_desc_mn_sw128(a + kk * 2048, BK * 128) : smem_desc_sw128(a + kk * 32);
                    };
                    auto desc_b = [&](uint32_t b, int kk) {
                        return B_MN ? smem_desc_mn_sw128(b + kk * 2048, BK * 128) : smem_desc_sw128(b + kk * 32);
                    };
                    const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        mma_f16_pair(d, desc_a(a0, kk), desc_b(b0, kk), idesc, (kb | kk) != 0 ? 1u : 0u);
                        if constexpr (SPL >= 2) mma_f16_pair(d, desc_a(a1, kk), desc_b(b0, kk), idesc, 1u);
                        if constexpr (SPL == 3) mma_f16_pair(d, desc_a(a0, kk), desc_b(b1, kk), idesc, 1u);
                    }
                    mma_commit_pair(smem_u32(empty + s));
                    mma_commit_pair(empty1 + 8u * static_cast<uint32_t>(s));
                }
                mma_commit_pair(smem_u32(tfull + buf));
                mma_commit_pair(tfull1 + 8u * static_cast<uint32_t>(buf));
                ++ti;
            }
            // both buffers drained by both CTAs' epilogues before the accumulators are freed
            for (int i = 0; i < 2 && ok; ++i, ++ti)
                if (!mbar_wait(tempty + (ti & 1), ((ti >> 1) & 1) ^ 1, abort_flag, p.err)) ok = false;
        }
    } else {
        const int e = warp - 2;
        const int quarter = warp & 3;
        const int half = e >> 2;
        uint8_t* stage = sOut + e * C::STAGE_OUT;
        const uint32_t tempty0 = cluster_addr(tempty, 0);
        uint32_t ti = 0;
        for (int u = pair; u < pp.units; u += npairs) {
            const PairUnit w = pair_unit(pp, u, tiles_n, kchunk, kblocks);
            if (w.skip) continue;
            const int cols = w.wide ? BN / 2 : BN / 4;     // this warp's columns of the unit
            const int buf = ti & 1;
            const int m0 = w.m0 + static_cast<int>(rank) * BM;
            int pos = -1;
            if constexpr (EPI == EPI_QKV) pos = qkv_rot_pos(p, m0 + quarter * 32 + lane, w.n0 + half * cols);
            if (!mbar_wait(tfull + buf, (ti >> 1) & 1, abort_flag, p.err)) break;
            tc_fence_after();
            const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN + half * cols);
            if constexpr (EPI == EPI_QKV)
                drain_qkv(tbase, stage, &tmOut, &tmOut2, pp.has_lo != 0, p, w.first ? p.bias : nullptr, w.n0 + half * cols,
                          m0 + quarter * 32, lane, cols, pos);
            else
                drain_rows<EPI>(tbase, stage, &tmOut, w.first ? p.bias : nullptr, p.N, w.n0 + half * cols,
                                m0 + quarter * 32, lane, cols);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + 8u * static_cast<uint32_t>(buf));
            ++ti;
        }
        if (lane == 0) bulk_wait_all();
    }

    // neither CTA leaves while the other may still arrive on its barriers or read its stages
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

template <int BN, int STAGES, int A_MN, int B_MN, int EPI>
static int launch(const Args& a, cudaStream_t stream) {
    using C = Cfg<BN, STAGES>;
    CUtensorMap tA, tB, tA2, tB2, tO;
    const int splits = a.A2 ? (a.B2 ? 3 : 2) : 1;   // passes (A, B), (A2, B), (A, B2)
    const bool split = splits > 1;
    auto map_a = [&](CUtensorMap* m, const void* ptr) {
        if (A_MN) return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.M, static_cast<uint64_t>(a.lda) * 2, BK, 64);
        return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, static_cast<uint64_t>(a.lda) * 2, BM, BK);
    };
    auto map_b = [&](CUtensorMap* m, const void* ptr) {
        if (B_MN) return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.N, static_cast<uint64_t>(a.ldb) * 2, BK, 64);
        return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, static_cast<uint64_t>(a.ldb) * 2, BN, BK);
    };
    int rc = map_a(&tA, a.A);
    if (!rc) rc = map_b(&tB, a.B);
    if (!rc) rc = map_a(&tA2, split ? a.A2 : a.A);
    if (!rc) rc = map_b(&tB2, splits == 3 ? a.B2 : a.B);
    if (!rc) {
        if (EPI == EPI_BF16)
            rc = make_tmap_2d(&tO, a.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.N, static_cast<uint64_t>(a.ldo) * 2, 32, 64, true);
        else
            rc = make_tmap_2d(&tO, a.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.M, a.N, static_cast<uint64_t>(a.ldo) * 4, 32, 32, true);
    }
    if (rc) return rc;
    auto kern = gemm_bf16_kernel<BN, STAGES, A_MN, B_MN, EPI>;
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    static DeviceOnce attr;   // per instantiation
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr.mark(dev);
    }
    int nsm = 0;
    if (int e = sm_count(dev, &nsm)) return e;
    const int tiles = ((a.N + BN - 1) / BN) * ((a.M + BM - 1) / BM);
    // an accumulating product may split K (ksplit.h: few output tiles over a long K)
    const int ksplit = EPI == EPI_F32_ADD && a.ksplit_ok ? choose_ksplit(tiles, (a.K + BK - 1) / BK, nsm) : 1;
    const int units = tiles * ksplit;
    KParams p{a.M, a.N, a.K, splits, ksplit, a.bias, a.err};
    kern<<<units < nsm ? units : nsm, C::THREADS, C::SMEM, stream>>>(tA, tB, tA2, tB2, tO, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

// The pair kernel's launch: grid = 2 × (pairs resident at once, at most the work units), 74 pairs on 148 SMs.
template <int STAGES, int SPL, int A_MN, int B_MN, int EPI>
static int launch_pair(const Args& a, cudaStream_t stream) {
    using C = PairCfg<STAGES, SPL>;
    CUtensorMap tA, tB, tA2, tB2, tBn, tB2n, tO;
    const int splits = a.A2 ? (a.B2 ? 3 : 2) : 1;
    const bool split = splits > 1;
    auto map_a = [&](CUtensorMap* m, const void* ptr) {
        if (A_MN) return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.M, static_cast<uint64_t>(a.lda) * 2, BK, 64);
        return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, static_cast<uint64_t>(a.lda) * 2, BM, BK);
    };
    // each CTA loads `rows` of the unit's B rows: 128 of a 256-wide unit, 64 of a narrow one (an N-contiguous B is
    // loaded as 64-column boxes either way)
    auto map_b = [&](CUtensorMap* m, const void* ptr, uint32_t rows) {
        if (B_MN) return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.N, static_cast<uint64_t>(a.ldb) * 2, BK, 64);
        return make_tmap_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, static_cast<uint64_t>(a.ldb) * 2, rows, BK);
    };
    const void* b2 = splits == 3 ? a.B2 : a.B;
    int rc = map_a(&tA, a.A);
    if (!rc) rc = map_b(&tB, a.B, PAIR_BN / 2);
    if (!rc) rc = map_a(&tA2, split ? a.A2 : a.A);
    if (!rc) rc = map_b(&tB2, b2, PAIR_BN / 2);
    if (!rc) rc = map_b(&tBn, a.B, PAIR_BN / 4);
    if (!rc) rc = map_b(&tB2n, b2, PAIR_BN / 4);
    CUtensorMap tO2;
    if (!rc) {
        if (EPI == EPI_BF16 || EPI == EPI_QKV)
            rc = make_tmap_2d(&tO, a.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.N, static_cast<uint64_t>(a.ldo) * 2, 32, 64, true);
        else
            rc = make_tmap_2d(&tO, a.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.M, a.N, static_cast<uint64_t>(a.ldo) * 4, 32, 32, true);
    }
    if (!rc) {
        if (EPI == EPI_QKV && a.out2)
            rc = make_tmap_2d(&tO2, a.out2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.N, static_cast<uint64_t>(a.ldo) * 2, 32, 64, true);
        else
            tO2 = tO;
    }
    if (rc) return rc;
    auto kern = gemm_bf16_pair_kernel<STAGES, SPL, A_MN, B_MN, EPI>;
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    static DeviceOnce attr;
    static std::atomic<int> resident[64];   // pairs resident at once, per device
    int pairs = dev >= 0 && dev < 64 ? resident[dev].load(std::memory_order_relaxed) : 0;
    if (!attr.done(dev) || pairs <= 0) {
        LAYA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        int nsm = 0;
        if (int e = sm_count(dev, &nsm)) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(nsm & ~1);
        cfg.blockDim = dim3(C::THREADS);
        cfg.dynamicSmemBytes = C::SMEM;
        LAYA_CUDA(cudaOccupancyMaxActiveClusters(&pairs, kern, &cfg));
        if (pairs <= 0) { set_error("the bf16 pair product cannot place a cluster of two CTAs"); return ERR_CUDA; }
        pairs = std::min(pairs, nsm / 2);
        if (dev >= 0 && dev < 64) resident[dev].store(pairs, std::memory_order_relaxed);
        attr.mark(dev);
    }
    const int tiles = ((a.N + PAIR_BN - 1) / PAIR_BN) * ((a.M + 2 * BM - 1) / (2 * BM));
    const int ksplit = EPI == EPI_F32_ADD && a.ksplit_ok ? choose_ksplit(tiles, (a.K + BK - 1) / BK, pairs) : 1;
    PairParams pp{KParams{a.M, a.N, a.K, splits, ksplit, a.bias, a.err, a.tok_item, a.seg_start, a.cosv, a.sinv,
                          a.rot_cols},
                  tiles * ksplit, tiles * ksplit, a.out2 ? 1 : 0};
    const int rem = tiles % pairs;
    if (ksplit == 1 && rem > 0 && 2 * rem <= pairs) {   // the last partial round, split along N
        pp.split_from = tiles - rem;
        pp.units = pp.split_from + 2 * rem;
    }
    kern<<<2 * std::min(pp.units, pairs), C::THREADS, C::SMEM, stream>>>(tA, tB, tA2, tB2, tBn, tB2n, tO, tO2, pp);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

template <int STAGES, int SPL, int EPI>
static int dispatch_pair_major(const Args& a, cudaStream_t s) {
    if (!a.a_mn && !a.b_mn) return launch_pair<STAGES, SPL, 0, 0, EPI>(a, s);
    if (!a.a_mn && a.b_mn) return launch_pair<STAGES, SPL, 0, 1, EPI>(a, s);
    if (a.a_mn && a.b_mn) return launch_pair<STAGES, SPL, 1, 1, EPI>(a, s);
    return launch_pair<STAGES, SPL, 1, 0, EPI>(a, s);
}

// stages per operand set: 6 × 32 KB plain, 4 × 48 KB with A's low part, 3 × 64 KB with both low parts
template <int EPI>
static int dispatch_pair(const Args& a, cudaStream_t s) {
    if (a.A2 && a.B2) return dispatch_pair_major<3, 3, EPI>(a, s);
    if (a.A2) return dispatch_pair_major<4, 2, EPI>(a, s);
    return dispatch_pair_major<6, 1, EPI>(a, s);
}

template <int BN, int STAGES, int EPI>
static int dispatch_major(const Args& a, cudaStream_t s) {
    if (!a.a_mn && !a.b_mn) return launch<BN, STAGES, 0, 0, EPI>(a, s);
    if (!a.a_mn && a.b_mn) return launch<BN, STAGES, 0, 1, EPI>(a, s);
    if (a.a_mn && a.b_mn) return launch<BN, STAGES, 1, 1, EPI>(a, s);
    return launch<BN, STAGES, 1, 0, EPI>(a, s);
}

// Products with N > 128 and more than one 128-row tile run on CTA pairs unless LAYA_GEMM_PAIR=0 is set in the
// environment (read once), which keeps the one-CTA 128 × 256 kernel: a diagnostic for comparing the two forms.
static bool pair_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("LAYA_GEMM_PAIR");
        return !(v && v[0] == '0');
    }();
    return on;
}

int gemm(const Args& a, cudaStream_t stream) {
    if (a.M <= 0 || a.N <= 0) return OK;
    if (a.K <= 0) { set_error("bf16 product needs K > 0"); return ERR_ARGUMENT; }
    if (a.B2 && !a.A2) { set_error("a split product with a low part of B needs the low part of A"); return ERR_ARGUMENT; }
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B) | reinterpret_cast<uintptr_t>(a.out) |
                         reinterpret_cast<uintptr_t>(a.A2) | reinterpret_cast<uintptr_t>(a.B2);
    if ((al & 15) || (a.lda & 7) || (a.ldb & 7) || ((a.epi == EPI_BF16 || a.epi == EPI_QKV) ? (a.ldo & 7) : (a.ldo & 3))) {
        set_error("bf16 product operands need 16-byte aligned bases and row strides");
        return ERR_ARGUMENT;
    }
    if (a.epi == EPI_QKV) {   // CTA pairs only, operands K-major, 64-column heads; the caller falls back otherwise
        if (a.N <= 128 || a.M <= BM || !pair_enabled() || a.a_mn || a.b_mn || (a.N % 64) || (a.rot_cols % 64) ||
            (reinterpret_cast<uintptr_t>(a.out2) & 15) || (a.cosv && (!a.sinv || !a.tok_item || !a.seg_start)) ||
            (reinterpret_cast<uintptr_t>(a.cosv) & 15) || (reinterpret_cast<uintptr_t>(a.sinv) & 15))
            return ERR_NOT_SUPPORTED;
        if (a.A2 && a.B2) return launch_pair<3, 3, 0, 0, EPI_QKV>(a, stream);
        if (a.A2) return launch_pair<4, 2, 0, 0, EPI_QKV>(a, stream);
        return launch_pair<6, 1, 0, 0, EPI_QKV>(a, stream);
    }
    if (a.N <= 128) {
        switch (a.epi) {
            case EPI_BF16: return dispatch_major<128, 4, EPI_BF16>(a, stream);
            case EPI_F32: return dispatch_major<128, 4, EPI_F32>(a, stream);
            case EPI_F32_ADD: return dispatch_major<128, 4, EPI_F32_ADD>(a, stream);
        }
    } else if (a.M > BM && pair_enabled()) {
        switch (a.epi) {
            case EPI_BF16: return dispatch_pair<EPI_BF16>(a, stream);
            case EPI_F32: return dispatch_pair<EPI_F32>(a, stream);
            case EPI_F32_ADD: return dispatch_pair<EPI_F32_ADD>(a, stream);
        }
    } else {
        switch (a.epi) {
            case EPI_BF16: return dispatch_major<256, 4, EPI_BF16>(a, stream);
            case EPI_F32: return dispatch_major<256, 4, EPI_F32>(a, stream);
            case EPI_F32_ADD: return dispatch_major<256, 4, EPI_F32_ADD>(a, stream);
        }
    }
    set_error("unknown bf16 product epilogue");
    return ERR_ARGUMENT;
}

}  // namespace bf
}  // namespace laya
