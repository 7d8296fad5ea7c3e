// flash.cu — attention forward and backward of the training step (bf16 operands, fp32 softmax and accumulators).
//
// Replaces Ops.AttentionForward/ForwardUnit and Ops.AttentionBackward/BackwardUnit with Rotary
// (Laya.Training/Ops.cs:260-504):
//   * per (segment, head), positions restarting at 0 in every segment; sliding layers see [i - W, i + W];
//   * rotary (rotate half) is applied once per layer by the prep pass (q and k at their segment positions, fp32
//     arithmetic as Rotary.Apply); the backward rotates dq and dk back (Rotary.Apply with inverse: true);
//   * dropout on the probabilities (the decision head's layers in training) by the reference's counter hash
//     Ops.Uniform(seed, (head << 42) | (row << 21) | key) with row the token's index in the batch and key the key's
//     position in its segment, so masks are the reference's bit for bit;
//   * forward keeps the row log-sum-exp; backward recomputes P from it:
//       D_i = Σ_d dO_id · O_id;  dP_ij = mask_ij · dO_i·v_j;  dS_ij = scale · P_ij · (dP_ij − D_i)
//       dV_j = Σ_i P_ij mask_ij dO_i;  dQ_i = Σ_j dS_ij k_j;  dK_j = Σ_i dS_ij q_i
//     split into a query-tile kernel (dQ) and a key-tile kernel (dK, dV), each recomputing P: no atomics, so the
//     gradients are deterministic.
// Tiles are 64 queries × 64 keys; each of the 4 warps owns 16 rows; mma.sync m16n8k16 bf16 → fp32.  The streamed
// operand (K/V in the forward and dQ kernels, Q/dO in the dK/dV kernel) is double-buffered with cp.async so the next
// tile lands while the current one is multiplied.
// The accurate forward (qkv_lo set) forms every product from bf16 hi/lo parts (three MMAs per product: scores and
// P·V) and writes the context as hi and lo; the backward reads the hi parts.
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "train.h"

namespace laya {
namespace fa {

constexpr int T64 = 64;
constexpr int LDS = 64 + 8;   // smem row stride (bf16): 144 bytes, 16-byte aligned rows, ldmatrix conflict-free
constexpr int TILE = T64 * LDS;
constexpr float LOG2E = 1.4426950408889634f;

DEVI void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
DEVI void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
DEVI void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
DEVI uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Ops.Uniform (Ops.cs:227-234) on the device: the same 64-bit mixing, the same fp32 result.
DEVI float dropout_uniform(uint64_t seed, uint64_t index) {
    uint64_t z = seed + (index + 1ull) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}
DEVI float drop_mult(const Args& a, int head, int row, int key) {
    if (a.dropout <= 0.0f) return 1.0f;
    const uint64_t idx = (static_cast<uint64_t>(head) << 42) | (static_cast<uint64_t>(row) << 21) | static_cast<uint32_t>(key);
    return dropout_uniform(a.seed, idx) < a.dropout ? 0.0f : a.keep;
}

DEVI void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
DEVI void cp_async4(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}
DEVI void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
DEVI void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 64 rows × HD bf16 at segment positions [p0, p0 + 64) of a [T, ld] buffer into a [64][LDS] smem tile; rows at or
// past `limit` are zero-filled (their source address is the segment's first row, never read).
template <int HD>
DEVI void cp_tile(__nv_bfloat16* dst, const __nv_bfloat16* base, int ld, int p0, int limit) {
    constexpr int CH = HD / 8;
    for (int it = threadIdx.x; it < T64 * CH; it += blockDim.x) {
        const int r = it / CH, c = it % CH;
        const bool ok = p0 + r < limit;
        const __nv_bfloat16* src = base + (ok ? static_cast<size_t>(p0 + r) * ld : 0) + c * 8;
        cp_async16(smem_u32(dst + r * LDS + c * 8), src, ok);
    }
}

// fp32 / bf16 quads
DEVI void load4(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 f = __bfloat1622float2(h[0]);
    v[0] = f.x; v[1] = f.y;
    f = __bfloat1622float2(h[1]);
    v[2] = f.x; v[3] = f.y;
}
DEVI void load4(const float* p, float (&v)[4]) {
    const float4 f = *reinterpret_cast<const float4*>(p);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
}
DEVI uint2 pack4(const float (&v)[4]) { return make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3])); }
DEVI uint2 pack4_lo(const float (&v)[4]) {
    float r[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) r[t] = v[t] - __bfloat162float(__float2bfloat16_rn(v[t]));
    return pack4(r);
}

// ------------------------------------------------------------------------------------------------ prep
// q and k rotated at their segment positions (Rotary.Apply, Ops.cs:490-503, fp32), v copied; from fp32 or bf16
// [T, lds]; to bf16 hi [T, ldd] (+ the low parts in the accurate forward).  One thread per 4 rotation pairs.  In place
// (src == hi, bf16) is allowed: a thread writes only what it read.
template <int HD, typename Src>
__global__ void prep_kernel(const Src* src, int lds, int T, int hidden, int heads, const int32_t* __restrict__ tok_item,
                            const int32_t* __restrict__ seg_start, const float* __restrict__ cosv,
                            const float* __restrict__ sinv, __nv_bfloat16* hi, __nv_bfloat16* __restrict__ lo, int ldd) {
    constexpr int HALF = HD / 2, J = HALF / 4;
    const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<size_t>(T) * heads * 3 * J) return;
    const int j = static_cast<int>(idx % J);
    size_t rest = idx / J;
    const int part = static_cast<int>(rest % 3);
    rest /= 3;
    const int h = static_cast<int>(rest % heads);
    const int t = static_cast<int>(rest / heads);
    const int col = part * hidden + h * HD + 4 * j;
    float a[4], b[4];
    load4(src + static_cast<size_t>(t) * lds + col, a);
    load4(src + static_cast<size_t>(t) * lds + col + HALF, b);
    if (part < 2 && cosv) {
        const int pos = t - seg_start[tok_item[t]];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float c = cosv[static_cast<size_t>(pos) * HALF + 4 * j + e];
            const float s = sinv[static_cast<size_t>(pos) * HALF + 4 * j + e];
            const float x = a[e], y = b[e];
            a[e] = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
            b[e] = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, s));
        }
    }
    __nv_bfloat16* d = hi + static_cast<size_t>(t) * ldd + col;
    *reinterpret_cast<uint2*>(d) = pack4(a);
    *reinterpret_cast<uint2*>(d + HALF) = pack4(b);
    if (lo) {
        __nv_bfloat16* l = lo + static_cast<size_t>(t) * ldd + col;
        *reinterpret_cast<uint2*>(l) = pack4_lo(a);
        *reinterpret_cast<uint2*>(l + HALF) = pack4_lo(b);
    }
}

// Q fragments (A operand) of the warp's 16 rows from a [64][LDS] smem tile.
template <int KS>
DEVI void load_a_frags(const __nv_bfloat16* tile, int warp, int lane, uint32_t (&fa)[KS][4]) {
    const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
        ldsm_x4(smem_u32(tile + r * LDS + ks * 16 + 8 * (lane >> 4)), fa[ks][0], fa[ks][1], fa[ks][2], fa[ks][3]);
}

// acc[16 rows x 64 cols] += A(16 x HD frags) · Bᵀ where B rows are the 64 smem rows (B[k=d][n=row] = tile[row][d]).
template <int KS>
DEVI void mma_abt(float (&acc)[8][4], const uint32_t (&fa)[KS][4], const __nv_bfloat16* tile, int lane) {
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
            const int row = jp * 16 + (lane & 7) + 8 * (lane >> 4);
            const int col = ks * 16 + 8 * ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(smem_u32(tile + row * LDS + col), b0, b1, b2, b3);
            mma_bf16(acc[2 * jp], fa[ks][0], fa[ks][1], fa[ks][2], fa[ks][3], b0, b1);
            mma_bf16(acc[2 * jp + 1], fa[ks][0], fa[ks][1], fa[ks][2], fa[ks][3], b2, b3);
        }
    }
}

// out[16 x HD] += P(16 x 64, as packed A frags from C frags) · tile(64 rows x HD)   (B[k=row][n=d] = tile[row][d])
template <int NT>
DEVI void mma_pv(float (&out)[NT][4], const uint32_t (&pa)[8][2], const __nv_bfloat16* tile, int lane) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int dp = 0; dp < NT / 2; ++dp) {
            const int row = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
            const int col = dp * 16 + 8 * (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(smem_u32(tile + row * LDS + col), b0, b1, b2, b3);
            mma_bf16(out[2 * dp], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b0, b1);
            mma_bf16(out[2 * dp + 1], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b2, b3);
        }
    }
}

DEVI bool visible(bool global, int W, int q, int k, int L) { return k < L && q < L && (global || (k >= q - W && k <= q + W)); }

// ------------------------------------------------------------------------------------------------ forward
// SPLIT (the accurate forward): scores = qh·kh + ql·kh + qh·kl, context = Ph·vh + Pl·vh + Ph·vl, written as hi and lo.
template <int HD, bool SPLIT>
__global__ void __launch_bounds__(128) fwd_kernel(Args a) {
    constexpr int KS = HD / 16, NT = HD / 8;
    constexpr int NQ = SPLIT ? 2 : 1, NB = SPLIT ? 4 : 2;   // Q tiles; tiles per K/V stage (K, V, K lo, V lo)
    extern __shared__ __align__(16) __nv_bfloat16 fsm[];
    __nv_bfloat16* Qs = fsm;
    __nv_bfloat16* stage0 = fsm + NQ * TILE;
    const int tile = blockIdx.x;
    if (tile >= *a.n_tiles) return;
    const int head = blockIdx.y, item = a.tile_item[tile], q0 = a.tile_p0[tile];
    const int seg0 = a.seg_start[item], L = a.seg_len[item];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const bool global = a.window < 0;
    const int W = a.window;
    const __nv_bfloat16* qb = a.qkv + static_cast<size_t>(seg0) * a.ld + head * HD;
    const __nv_bfloat16* lb = SPLIT ? a.qkv_lo + static_cast<size_t>(seg0) * a.ld + head * HD : nullptr;
    const int kb = global ? 0 : max(0, q0 - W), ke = global ? L : min(L, q0 + T64 + W);
    const int nk = (ke - kb + T64 - 1) / T64;
    auto load_kv = [&](int j) {
        __nv_bfloat16* d = stage0 + (j & 1) * NB * TILE;
        const int k0 = kb + j * T64;
        cp_tile<HD>(d, qb + a.hidden, a.ld, k0, ke);
        cp_tile<HD>(d + TILE, qb + 2 * a.hidden, a.ld, k0, ke);
        if constexpr (SPLIT) {
            cp_tile<HD>(d + 2 * TILE, lb + a.hidden, a.ld, k0, ke);
            cp_tile<HD>(d + 3 * TILE, lb + 2 * a.hidden, a.ld, k0, ke);
        }
    };
    cp_tile<HD>(Qs, qb, a.ld, q0, L);
    if constexpr (SPLIT) cp_tile<HD>(Qs + TILE, lb, a.ld, q0, L);
    load_kv(0);
    cp_commit();
    uint32_t fq[KS][4], fql[SPLIT ? KS : 1][4];
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const int qp[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};
    for (int jt = 0; jt < nk; ++jt) {
        if (jt + 1 < nk) {
            load_kv(jt + 1);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        if (jt == 0) {
            load_a_frags<KS>(Qs, warp, lane, fq);
            if constexpr (SPLIT) load_a_frags<KS>(Qs + TILE, warp, lane, fql);
        }
        const __nv_bfloat16* Ks = stage0 + (jt & 1) * NB * TILE;
        const __nv_bfloat16* Vs = Ks + TILE;
        const int k0 = kb + jt * T64;
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
        mma_abt<KS>(s, fq, Ks, lane);
        if constexpr (SPLIT) {
            mma_abt<KS>(s, fql, Ks, lane);
            mma_abt<KS>(s, fq, Ks + 2 * TILE, lane);
        }
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int kp = k0 + 8 * j + 2 * t4 + (e & 1);
                const float v = visible(global, W, qp[e >> 1], kp, ke) ? __fmul_rn(s[j][e], a.scale) : -INFINITY;
                s[j][e] = v;
                mx[e >> 1] = fmaxf(mx[e >> 1], v);
            }
        float alpha[2], msc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
            const float mn = fmaxf(m_run[h], mx[h]);
            alpha[h] = m_run[h] == -INFINITY ? 0.f : exp2f((m_run[h] - mn) * LOG2E);
            msc[h] = mn * LOG2E;
            m_run[h] = mn;
        }
        float rs[2] = {0.f, 0.f};
        uint32_t pa[8][2], pl[SPLIT ? 8 : 1][2];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float pv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1;
                const float pe = s[j][e] == -INFINITY ? 0.f : exp2f(fmaf(s[j][e], LOG2E, -msc[h]));
                rs[h] += pe;   // the normaliser counts every probability, dropped or not
                const int kp = k0 + 8 * j + 2 * t4 + (e & 1);
                pv[e] = pe == 0.f ? 0.f : pe * drop_mult(a, head, seg0 + qp[h], kp);
            }
            pa[j][0] = pack_bf16(pv[0], pv[1]);
            pa[j][1] = pack_bf16(pv[2], pv[3]);
            if constexpr (SPLIT) {
                const uint2 r = pack4_lo(pv);
                pl[j][0] = r.x;
                pl[j][1] = r.y;
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
            l_run[h] = l_run[h] * alpha[h] + rs[h];
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) { o[j][0] *= alpha[0]; o[j][1] *= alpha[0]; o[j][2] *= alpha[1]; o[j][3] *= alpha[1]; }
        mma_pv<NT>(o, pa, Vs, lane);
        if constexpr (SPLIT) {
            mma_pv<NT>(o, pl, Vs, lane);
            mma_pv<NT>(o, pa, Ks + 3 * TILE, lane);
        }
        __syncthreads();   // this stage is refilled by the prefetch two tiles on
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int q = qp[h];
        if (q >= L) continue;
        const float inv = l_run[h] > 0.f ? 1.0f / l_run[h] : 0.f;
        __nv_bfloat16* orow = a.out + static_cast<size_t>(seg0 + q) * a.ldo + head * HD;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const float c0 = o[j][2 * h] * inv, c1 = o[j][2 * h + 1] * inv;
            *reinterpret_cast<uint32_t*>(orow + 8 * j + 2 * t4) = pack_bf16(c0, c1);
            if constexpr (SPLIT) {
                __nv_bfloat16* lrow = a.out_lo + static_cast<size_t>(seg0 + q) * a.ldo + head * HD;
                *reinterpret_cast<uint32_t*>(lrow + 8 * j + 2 * t4) =
                    pack_bf16(c0 - __bfloat162float(__float2bfloat16_rn(c0)), c1 - __bfloat162float(__float2bfloat16_rn(c1)));
            }
        }
        if (t4 == 0) a.lse[static_cast<size_t>(seg0 + q) * a.heads + head] = m_run[h] + logf(l_run[h]);
    }
}

// D_i = Σ_d dO · O per (token, head), fp32.  HD/8 lanes per (token, head), each reading 8 consecutive bf16 of dO
// and O with one 16-byte load apiece, then a shuffle sum over the group; a thread takes DOT_ROWS tokens T/DOT_ROWS
// apart, with every load issued before the first sum.
constexpr int DOT_ROWS = 4;
template <int HD>
__global__ void bwd_dot_kernel(Args a, int T) {
    constexpr int G = HD / 8;   // lanes per (token, head)
    const int per = (T + DOT_ROWS - 1) / DOT_ROWS;   // tokens per slice
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    const int item = gt / G, l = gt % G;
    const bool active = item < per * a.heads;
    const int it = active ? item : 0;
    const int t0 = it / a.heads, h = it % a.heads;
    uint4 x[DOT_ROWS], y[DOT_ROWS];
#pragma unroll
    for (int r = 0; r < DOT_ROWS; ++r) {
        const int t = t0 + r * per;
        const size_t off = static_cast<size_t>(t < T ? t : 0) * a.ldo + h * HD + 8 * l;
        x[r] = *reinterpret_cast<const uint4*>(a.dout + off);
        y[r] = *reinterpret_cast<const uint4*>(a.out + off);
    }
#pragma unroll
    for (int r = 0; r < DOT_ROWS; ++r) {
        const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&x[r]);
        const __nv_bfloat162* ya = reinterpret_cast<const __nv_bfloat162*>(&y[r]);
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 u = __bfloat1622float2(xa[k]), v = __bfloat1622float2(ya[k]);
            s = fmaf(u.x, v.x, s);
            s = fmaf(u.y, v.y, s);
        }
#pragma unroll
        for (int m = G / 2; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
        const int t = t0 + r * per;
        if (active && l == 0 && t < T) a.dsum[static_cast<size_t>(t) * a.heads + h] = s;
    }
}

// Writes 16 rows x HD of a warp's fp32 accumulator as bf16 into a [T, ld] slice, rotating back by -θ when given.
template <int NT>
DEVI void store_rows(float (&acc)[NT][4], __nv_bfloat16* base, int ld, int seg0, int p0, int warp, int lane, int L,
                     const float* cosv, const float* sinv) {
    constexpr int HD = NT * 8, HALF = HD / 2;
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int pos = p0 + warp * 16 + g + 8 * h;
        if (cosv) {
            // pairs (i, i + HALF) live in n-tiles j and j + NT/2 of the same thread
#pragma unroll
            for (int j = 0; j < NT / 2; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int i = 8 * j + 2 * t4 + e;
                    const float c = pos < L ? cosv[static_cast<size_t>(pos) * HALF + i] : 0.f;
                    const float s = pos < L ? sinv[static_cast<size_t>(pos) * HALF + i] : 0.f;
                    const float x = acc[j][2 * h + e], y = acc[j + NT / 2][2 * h + e];
                    acc[j][2 * h + e] = __fadd_rn(__fmul_rn(x, c), __fmul_rn(y, s));
                    acc[j + NT / 2][2 * h + e] = __fsub_rn(__fmul_rn(y, c), __fmul_rn(x, s));
                }
        }
        if (pos < L) {
            __nv_bfloat16* row = base + static_cast<size_t>(seg0 + pos) * ld;
#pragma unroll
            for (int j = 0; j < NT; ++j)
                *reinterpret_cast<uint32_t*>(row + 8 * j + 2 * t4) = pack_bf16(acc[j][2 * h], acc[j][2 * h + 1]);
        }
    }
}

// dQ for one 64-query tile of one head; K/V tiles double-buffered.
template <int HD>
__global__ void __launch_bounds__(128) bwd_dq_kernel(Args a) {
    constexpr int KS = HD / 16, NT = HD / 8;
    extern __shared__ __align__(16) __nv_bfloat16 fsm[];
    __nv_bfloat16* Qs = fsm;
    __nv_bfloat16* dOs = fsm + TILE;
    __nv_bfloat16* stage0 = fsm + 2 * TILE;   // [2][K, V]
    const int tile = blockIdx.x;
    if (tile >= *a.n_tiles) return;
    const int head = blockIdx.y, item = a.tile_item[tile], q0 = a.tile_p0[tile];
    const int seg0 = a.seg_start[item], L = a.seg_len[item];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const bool global = a.window < 0;
    const int W = a.window;
    const __nv_bfloat16* qb = a.qkv + static_cast<size_t>(seg0) * a.ld + head * HD;
    const int kb = global ? 0 : max(0, q0 - W), ke = global ? L : min(L, q0 + T64 + W);
    const int nk = (ke - kb + T64 - 1) / T64;
    auto load_kv = [&](int j) {
        __nv_bfloat16* d = stage0 + (j & 1) * 2 * TILE;
        cp_tile<HD>(d, qb + a.hidden, a.ld, kb + j * T64, ke);
        cp_tile<HD>(d + TILE, qb + 2 * a.hidden, a.ld, kb + j * T64, ke);
    };
    cp_tile<HD>(Qs, qb, a.ld, q0, L);
    cp_tile<HD>(dOs, a.dout + static_cast<size_t>(seg0) * a.ldo + head * HD, a.ldo, q0, L);
    load_kv(0);
    cp_commit();
    const int qp[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};
    float lse[2], dd[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const bool ok = qp[h] < L;
        lse[h] = ok ? a.lse[static_cast<size_t>(seg0 + qp[h]) * a.heads + head] : 0.f;
        dd[h] = ok ? a.dsum[static_cast<size_t>(seg0 + qp[h]) * a.heads + head] : 0.f;
    }
    uint32_t fq[KS][4], fdo[KS][4];
    float dq[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) dq[j][0] = dq[j][1] = dq[j][2] = dq[j][3] = 0.f;
    for (int jt = 0; jt < nk; ++jt) {
        if (jt + 1 < nk) {
            load_kv(jt + 1);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        if (jt == 0) {
            load_a_frags<KS>(Qs, warp, lane, fq);
            load_a_frags<KS>(dOs, warp, lane, fdo);
        }
        const __nv_bfloat16* Ks = stage0 + (jt & 1) * 2 * TILE;
        const __nv_bfloat16* Vs = Ks + TILE;
        const int k0 = kb + jt * T64;
        float s[8][4], dp[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[j][e] = dp[j][e] = 0.f;
        mma_abt<KS>(s, fq, Ks, lane);
        mma_abt<KS>(dp, fdo, Vs, lane);
        uint32_t pa[8][2];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float ds[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1;
                const int kp = k0 + 8 * j + 2 * t4 + (e & 1);
                float p = 0.f;
                if (visible(global, W, qp[h], kp, ke)) p = __expf(__fmul_rn(s[j][e], a.scale) - lse[h]);
                const float dpm = dp[j][e] * drop_mult(a, head, seg0 + qp[h], kp);
                ds[e] = a.scale * p * (dpm - dd[h]);
            }
            pa[j][0] = pack_bf16(ds[0], ds[1]);
            pa[j][1] = pack_bf16(ds[2], ds[3]);
        }
        mma_pv<NT>(dq, pa, Ks, lane);
        __syncthreads();
    }
    store_rows<NT>(dq, a.dqkv + head * HD, a.lddq, seg0, q0, warp, lane, L, a.cosv, a.sinv);
}

// dK and dV for one 64-key tile of one head; Q/dO tiles (with their rows' lse and D) double-buffered.
template <int HD>
__global__ void __launch_bounds__(128) bwd_dkdv_kernel(Args a) {
    constexpr int KS = HD / 16, NT = HD / 8;
    extern __shared__ __align__(16) __nv_bfloat16 fsm[];
    __nv_bfloat16* Ks = fsm;
    __nv_bfloat16* Vs = fsm + TILE;
    __nv_bfloat16* stage0 = fsm + 2 * TILE;                            // [2][Q, dO]
    float* rows0 = reinterpret_cast<float*>(fsm + 6 * TILE);          // [2][lse 64, D 64]
    const int tile = blockIdx.x;
    if (tile >= *a.n_tiles) return;
    const int head = blockIdx.y, item = a.tile_item[tile], k0 = a.tile_p0[tile];
    const int seg0 = a.seg_start[item], L = a.seg_len[item];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const bool global = a.window < 0;
    const int W = a.window;
    const __nv_bfloat16* qb = a.qkv + static_cast<size_t>(seg0) * a.ld + head * HD;
    const __nv_bfloat16* ob = a.dout + static_cast<size_t>(seg0) * a.ldo + head * HD;
    const int qb0 = global ? 0 : max(0, k0 - W), qe = global ? L : min(L, k0 + T64 + W);
    const int nq = (qe - qb0 + T64 - 1) / T64;
    auto load_q = [&](int j) {
        __nv_bfloat16* d = stage0 + (j & 1) * 2 * TILE;
        float* rr = rows0 + (j & 1) * 2 * T64;
        const int q0 = qb0 + j * T64;
        cp_tile<HD>(d, qb, a.ld, q0, qe);
        cp_tile<HD>(d + TILE, ob, a.ldo, q0, qe);
        for (int r = threadIdx.x; r < T64; r += blockDim.x) {
            const bool ok = q0 + r < qe;
            const size_t at = ok ? static_cast<size_t>(seg0 + q0 + r) * a.heads + head : 0;
            cp_async4(smem_u32(rr + r), a.lse + at, ok);
            cp_async4(smem_u32(rr + T64 + r), a.dsum + at, ok);
        }
    };
    cp_tile<HD>(Ks, qb + a.hidden, a.ld, k0, L);
    cp_tile<HD>(Vs, qb + 2 * a.hidden, a.ld, k0, L);
    load_q(0);
    cp_commit();
    uint32_t fk[KS][4], fv[KS][4];
    const int kp[2] = {k0 + warp * 16 + g, k0 + warp * 16 + g + 8};
    float dk[NT][4], dv[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) dk[j][e] = dv[j][e] = 0.f;
    for (int jt = 0; jt < nq; ++jt) {
        if (jt + 1 < nq) {
            load_q(jt + 1);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        if (jt == 0) {
            load_a_frags<KS>(Ks, warp, lane, fk);
            load_a_frags<KS>(Vs, warp, lane, fv);
        }
        const __nv_bfloat16* Qs = stage0 + (jt & 1) * 2 * TILE;
        const __nv_bfloat16* dOs = Qs + TILE;
        const float* lse_s = rows0 + (jt & 1) * 2 * T64;
        const float* dd_s = lse_s + T64;
        const int q0 = qb0 + jt * T64;
        // transposed scores: rows = this warp's 16 keys, columns = 64 queries
        float st[8][4], dpt[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) st[j][e] = dpt[j][e] = 0.f;
        mma_abt<KS>(st, fk, Qs, lane);
        mma_abt<KS>(dpt, fv, dOs, lane);
        uint32_t pm[8][2], dsa[8][2];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float pd[4], ds[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1;
                const int qr = 8 * j + 2 * t4 + (e & 1);
                const int q = q0 + qr;
                float p = 0.f;
                if (visible(global, W, q, kp[h], qe)) p = __expf(__fmul_rn(st[j][e], a.scale) - lse_s[qr]);
                const float m = drop_mult(a, head, seg0 + q, kp[h]);
                pd[e] = p * m;
                ds[e] = a.scale * p * (dpt[j][e] * m - dd_s[qr]);
            }
            pm[j][0] = pack_bf16(pd[0], pd[1]);
            pm[j][1] = pack_bf16(pd[2], pd[3]);
            dsa[j][0] = pack_bf16(ds[0], ds[1]);
            dsa[j][1] = pack_bf16(ds[2], ds[3]);
        }
        mma_pv<NT>(dv, pm, dOs, lane);
        mma_pv<NT>(dk, dsa, Qs, lane);
        __syncthreads();
    }
    store_rows<NT>(dk, a.dqkv + a.hidden + head * HD, a.lddq, seg0, k0, warp, lane, L, a.cosv, a.sinv);
    store_rows<NT>(dv, a.dqkv + 2 * a.hidden + head * HD, a.lddq, seg0, k0, warp, lane, L, nullptr, nullptr);
}

}  // namespace fa

// ------------------------------------------------------------------------------------------------ launchers
template <class K>
static int set_smem(K kern, int bytes) {
    static thread_local std::vector<std::pair<const void*, int>> done;   // (kernel, device) already configured
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    for (auto& d : done)
        if (d.first == reinterpret_cast<const void*>(kern) && d.second == dev) return OK;
    LAYA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.push_back({reinterpret_cast<const void*>(kern), dev});
    return OK;
}

int attn_prep(const void* src, int src_f32, int lds, int T, int hidden, int heads, const int32_t* tok_item,
              const int32_t* seg_start, const float* cosv, const float* sinv, __nv_bfloat16* hi, __nv_bfloat16* lo,
              int ldd, cudaStream_t s) {
    if (T <= 0) return OK;
    const int hd = hidden / heads;
    const size_t n = static_cast<size_t>(T) * heads * 3 * (hd / 8);
    const unsigned g = static_cast<unsigned>((n + 255) / 256);
    if (hd == 64) {
        if (src_f32) fa::prep_kernel<64, float><<<g, 256, 0, s>>>(static_cast<const float*>(src), lds, T, hidden, heads, tok_item, seg_start, cosv, sinv, hi, lo, ldd);
        else fa::prep_kernel<64, __nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(src), lds, T, hidden, heads, tok_item, seg_start, cosv, sinv, hi, lo, ldd);
    } else if (hd == 32) {
        if (src_f32) fa::prep_kernel<32, float><<<g, 256, 0, s>>>(static_cast<const float*>(src), lds, T, hidden, heads, tok_item, seg_start, cosv, sinv, hi, lo, ldd);
        else fa::prep_kernel<32, __nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(src), lds, T, hidden, heads, tok_item, seg_start, cosv, sinv, hi, lo, ldd);
    } else {
        set_error("attention supports head_dim 32 and 64");
        return ERR_NOT_SUPPORTED;
    }
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

template <int HD, bool SPLIT>
static int launch_fwd(const fa::Args& a, int max_tiles, cudaStream_t s) {
    const int smem = (SPLIT ? 10 : 5) * fa::TILE * 2;
    int rc = set_smem(fa::fwd_kernel<HD, SPLIT>, smem);
    if (rc) return rc;
    fa::fwd_kernel<HD, SPLIT><<<dim3(max_tiles, a.heads), 128, smem, s>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int flash_forward(const fa::Args& a, int max_tiles, cudaStream_t s) {
    if (max_tiles <= 0) return OK;
    const int hd = a.hidden / a.heads;
    const bool split = a.qkv_lo != nullptr;
    if (split && !a.out_lo) { set_error("accurate attention needs the context's low part"); return ERR_ARGUMENT; }
    if (hd == 64) {   // the tcgen05 forwards (flash_pp.cu, flash_tc.cu) when the batch carries their tile lists
        int rc = flash_forward_pp(a, s);
        if (rc != ERR_NOT_SUPPORTED) return rc;
        rc = flash_forward_tc(a, s);
        if (rc != ERR_NOT_SUPPORTED) return rc;
        return split ? launch_fwd<64, true>(a, max_tiles, s) : launch_fwd<64, false>(a, max_tiles, s);
    }
    if (hd == 32) return split ? launch_fwd<32, true>(a, max_tiles, s) : launch_fwd<32, false>(a, max_tiles, s);
    set_error("attention supports head_dim 32 and 64");
    return ERR_NOT_SUPPORTED;
}

template <int HD>
static int launch_bwd(const fa::Args& a, int max_tiles, cudaStream_t s) {
    const int smem_dq = 6 * fa::TILE * 2, smem_kv = 6 * fa::TILE * 2 + 4 * fa::T64 * 4;
    int rc = set_smem(fa::bwd_dq_kernel<HD>, smem_dq);
    if (!rc) rc = set_smem(fa::bwd_dkdv_kernel<HD>, smem_kv);
    if (rc) return rc;
    dim3 grid(max_tiles, a.heads);
    if (HD == 64 && a.ds && (a.window < 0 || a.window % 64 == 0)) {
        // dK, dV first, leaving every dS tile in the scratch; then dQ = dS·K streams them (flash_tc.cu)
        rc = flash_backward_dkdv_tc(a, s);
        if (rc == OK) return flash_backward_dq_ds(a, s);
        if (rc != ERR_NOT_SUPPORTED) return rc;
    }
    fa::Args a0 = a;   // the kernels below recompute S and dP for dQ and store no dS
    a0.ds = nullptr;
    rc = HD == 64 ? flash_backward_dq_tc(a0, s) : ERR_NOT_SUPPORTED;   // dQ on the tensor cores (flash_tc.cu)
    if (rc == ERR_NOT_SUPPORTED) {
        fa::bwd_dq_kernel<HD><<<grid, 128, smem_dq, s>>>(a0);
        count_launch();
        LAYA_CUDA(cudaGetLastError());
    } else if (rc != OK) {
        return rc;
    }
    if (HD == 64) {   // dK, dV on the tensor cores (flash_tc.cu) when the batch carries its 128-row tile list
        rc = flash_backward_dkdv_tc(a0, s);
        if (rc != ERR_NOT_SUPPORTED) return rc;
    }
    fa::bwd_dkdv_kernel<HD><<<grid, 128, smem_kv, s>>>(a0);
    count_launch();
    return OK;
}

int flash_backward(const fa::Args& a, int max_tiles, int T, cudaStream_t s) {
    if (max_tiles <= 0 || T <= 0) return OK;
    const int hd = a.hidden / a.heads;
    const long long threads = static_cast<long long>((T + fa::DOT_ROWS - 1) / fa::DOT_ROWS) * a.heads * (hd / 8);
    if ((a.ldo & 7) || (reinterpret_cast<uintptr_t>(a.dout) & 15) || (reinterpret_cast<uintptr_t>(a.out) & 15)) {
        set_error("attention backward: dO and O need 16-byte aligned rows");
        return ERR_ARGUMENT;
    }
    if (hd == 64) fa::bwd_dot_kernel<64><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(a, T);
    else if (hd == 32) fa::bwd_dot_kernel<32><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(a, T);
    count_launch();
    int rc;
    if (hd == 64) rc = launch_bwd<64>(a, max_tiles, s);
    else if (hd == 32) rc = launch_bwd<32>(a, max_tiles, s);
    else { set_error("attention supports head_dim 32 and 64"); return ERR_NOT_SUPPORTED; }
    if (rc) return rc;
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace laya
