// train_kernels.cu — the memory-bound kernels of the training step.
//
//   ln_fwd / ln_bwd        Ops.LayerNorm / Ops.LayerNormBackward (Laya.Training/Ops.cs:103-186); the forward keeps the
//                          row mean and 1/std for the backward (the reference recomputes them in double).
//   geglu_fwd / geglu_bwd  the GeGLU of EncoderLayerForward and its backward (TrainableDecisionModel.cs:391-398, 564-579;
//                          Ops.GeluBackward, Ops.cs:194-218), exact-erf GELU.
//   masked ops             ReLU, inverted dropout (Ops.Dropout, Ops.cs:244-258, the reference's counter hash) and the
//                          residual adds of HeadLayerForward/Backward (TrainableDecisionModel.cs:428-468, 605-640).
//   colsum                 bias gradients db += Σ_rows dy (Ops.LinearBackward, Ops.cs:64-68).
//   scatters               embedding-row and type-embedding gradients (TrainableDecisionModel.cs:513-521, 538-548).
//   scorer                 the option scorer's Linear(h, 1) and its backward (TrainableDecisionModel.cs:313-331, 484-504).
//   adamw / sumsq          AdamW.Step and Gradients.ClipByGlobalNorm (AdamW.cs:29-130) over flat parameter buffers,
//                          refreshing the bf16 copies the products read.
// Every kernel moves each byte once with 16-byte accesses where the layout allows; a warp owns a row for row-wise ops.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "train.h"

namespace laya {
namespace tr {

DEVI float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

// Ops.Uniform on the device (same mixing as fa::dropout_uniform).
DEVI float uniform_hash(uint64_t seed, uint64_t index) {
    uint64_t z = seed + (index + 1ull) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}
DEVI float dmask(const Mask& m, size_t i) {
    if (m.p <= 0.0f) return 1.0f;
    return uniform_hash(m.seed, static_cast<uint64_t>(i)) < m.p ? 0.0f : m.keep;
}

// The derivative of exact GELU, Φ(u) + u·φ(u) (Ops.GeluBackward).
DEVI float gelu_grad(float x) {
    const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752f));
    const float pdf = 0.39894228040143268f * __expf(-0.5f * x * x);
    return cdf + x * pdf;
}
DEVI float gelu_exact(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// ------------------------------------------------------------------------------------------------ LayerNorm
// One warp per row; n <= 32·NPL.
template <int NPL>
__global__ void __launch_bounds__(256) ln_fwd_kernel(LnFwd a) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= a.rows) return;
    const int n = a.n;
    const float* src;
    if (a.table) {
        int id = a.ids[row];
        if (id < 0 || id >= a.vocab) { if (lane == 0) atomicExch(a.err, LAYA_DEV_ERR_BOUNDS); id = 0; }
        src = a.table + static_cast<size_t>(id) * n;
    } else {
        src = a.x + static_cast<size_t>(a.gather ? a.gather[row] : row) * n;
    }
    float v[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) { const int c = lane + 32 * i; v[i] = c < n ? src[c] : 0.f; }
    if (a.identity) {
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int c = lane + 32 * i;
            if (c >= n) continue;
            const __nv_bfloat16 hi = __float2bfloat16_rn(v[i]);
            a.y16[static_cast<size_t>(row) * n + c] = hi;
            if (a.y16lo) a.y16lo[static_cast<size_t>(row) * n + c] = __float2bfloat16_rn(v[i] - bf(hi));
        }
        return;
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) s += v[i];
    const float mean = warp_sum(s) / n;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) { const int c = lane + 32 * i; const float d = c < n ? v[i] - mean : 0.f; q += d * d; }
    const float rstd = rsqrtf(warp_sum(q) / n + a.eps);
    if (lane == 0) { a.mean[row] = mean; a.rstd[row] = rstd; }
    const float* te = a.temb ? a.temb + static_cast<size_t>(a.qtype[a.tok_item[row]]) * n : nullptr;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
        const int c = lane + 32 * i;
        if (c >= n) continue;
        float y = (v[i] - mean) * rstd * a.w[c];
        if (a.b) y += a.b[c];
        if (a.y16) {
            const __nv_bfloat16 hi = __float2bfloat16_rn(y);
            a.y16[static_cast<size_t>(row) * n + c] = hi;
            if (a.y16lo) a.y16lo[static_cast<size_t>(row) * n + c] = __float2bfloat16_rn(y - bf(hi));
        }
        if (a.y32) a.y32[static_cast<size_t>(row) * n + c] = te ? y + te[c] : y;
    }
}

// dx (+)= rstd·(g − mean(g) − x̂·mean(g·x̂)), g = dy·γ; dγ += Σ dy·x̂; dβ += Σ dy.  A CTA of 8 warps takes
// LN_ROWS rows, each lane owns columns lane + 32i, and the CTA adds its column partials to dγ/dβ once.
constexpr int LN_ROWS = 64;
template <int NPL>
__global__ void __launch_bounds__(256) ln_bwd_kernel(LnBwd a) {
    __shared__ float red[8][32 * NPL];   // column partials of the 8 warps, for dγ then dβ
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n = a.n;
    float pw[NPL], pb[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) pw[i] = pb[i] = 0.f;
    const int r0 = blockIdx.x * LN_ROWS;
    for (int rr = warp; rr < LN_ROWS; rr += 8) {
        const int r = r0 + rr;
        if (r >= a.rows) break;
        const int xr = a.gather ? a.gather[r] : r;
        const float mean = a.mean[r], rstd = a.rstd[r];
        float xh[NPL], g[NPL], dy[NPL];
        float sg = 0.f, sgx = 0.f;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int c = lane + 32 * i;
            if (c < n) {
                const float x = a.x[static_cast<size_t>(xr) * n + c];
                dy[i] = a.dy[static_cast<size_t>(r) * n + c];
                xh[i] = (x - mean) * rstd;
                g[i] = dy[i] * a.w[c];
            } else {
                dy[i] = xh[i] = g[i] = 0.f;
            }
            sg += g[i];
            sgx += g[i] * xh[i];
            pw[i] += dy[i] * xh[i];
            pb[i] += dy[i];
        }
        const float mg = warp_sum(sg) / n, mgx = warp_sum(sgx) / n;
        if (a.dx) {
#pragma unroll
            for (int i = 0; i < NPL; ++i) {
                const int c = lane + 32 * i;
                if (c >= n) continue;
                const float d = rstd * (g[i] - mg - xh[i] * mgx);
                float* dst = a.dx + static_cast<size_t>(a.scatter ? a.scatter[r] : r) * n + c;
                if (a.scatter) atomicAdd(dst, d);
                else *dst = a.accumulate ? *dst + d : d;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < NPL; ++i) red[warp][lane + 32 * i] = pw[i];
    __syncthreads();
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
        float sw = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sw += red[w][c];
        if (a.dw) atomicAdd(a.dw + c, sw);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NPL; ++i) red[warp][lane + 32 * i] = pb[i];
    __syncthreads();
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
        float sb = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sb += red[w][c];
        if (a.db) atomicAdd(a.db + c, sb);
    }
}

// float4 variants for n = 128·VPL: lane owns columns 4·lane + 128·i .. +3, 16-byte loads and stores throughout.
DEVI void st_bf16x4(__nv_bfloat16* hi, __nv_bfloat16* lo, size_t i, const float4& y) {
    __nv_bfloat162 h0 = __floats2bfloat162_rn(y.x, y.y), h1 = __floats2bfloat162_rn(y.z, y.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&h0);
    u.y = *reinterpret_cast<uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(hi + i) = u;
    if (lo) {
        const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
        __nv_bfloat162 l0 = __floats2bfloat162_rn(y.x - f0.x, y.y - f0.y), l1 = __floats2bfloat162_rn(y.z - f1.x, y.w - f1.y);
        u.x = *reinterpret_cast<uint32_t*>(&l0);
        u.y = *reinterpret_cast<uint32_t*>(&l1);
        *reinterpret_cast<uint2*>(lo + i) = u;
    }
}
DEVI float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

template <int VPL>
__global__ void __launch_bounds__(256) ln_fwd_vec_kernel(LnFwd a) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= a.rows) return;
    const int n = a.n;
    const float* src;
    if (a.table) {
        int id = a.ids[row];
        if (id < 0 || id >= a.vocab) { if (lane == 0) atomicExch(a.err, LAYA_DEV_ERR_BOUNDS); id = 0; }
        src = a.table + static_cast<size_t>(id) * n;
    } else {
        src = a.x + static_cast<size_t>(a.gather ? a.gather[row] : row) * n;
    }
    float4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = ld4(src + 4 * lane + 128 * i);
    const size_t o = static_cast<size_t>(row) * n + 4 * lane;
    if (a.identity) {
#pragma unroll
        for (int i = 0; i < VPL; ++i) st_bf16x4(a.y16, a.y16lo, o + 128 * i, v[i]);
        return;
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = warp_sum(s) / n;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const float d0 = v[i].x - mean, d1 = v[i].y - mean, d2 = v[i].z - mean, d3 = v[i].w - mean;
        q += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
    }
    const float rstd = rsqrtf(warp_sum(q) / n + a.eps);
    if (lane == 0) { a.mean[row] = mean; a.rstd[row] = rstd; }
    const float* te = a.temb ? a.temb + static_cast<size_t>(a.qtype[a.tok_item[row]]) * n : nullptr;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = 4 * lane + 128 * i;
        const float4 w = ld4(a.w + c);
        float4 y = make_float4((v[i].x - mean) * rstd * w.x, (v[i].y - mean) * rstd * w.y, (v[i].z - mean) * rstd * w.z,
                               (v[i].w - mean) * rstd * w.w);
        if (a.b) {
            const float4 b = ld4(a.b + c);
            y.x += b.x; y.y += b.y; y.z += b.z; y.w += b.w;
        }
        if (a.y16) st_bf16x4(a.y16, a.y16lo, o + 128 * i, y);
        if (a.y32) {
            if (te) {
                const float4 t = ld4(te + c);
                y.x += t.x; y.y += t.y; y.z += t.z; y.w += t.w;
            }
            *reinterpret_cast<float4*>(a.y32 + o + 128 * i) = y;
        }
    }
}

constexpr int LN_ROWS_V = 32;   // rows per CTA of the vector backward: 4 per warp
template <int VPL>
__global__ void __launch_bounds__(256) ln_bwd_vec_kernel(LnBwd a) {
    __shared__ __align__(16) float red[8][128 * VPL];   // column partials of the 8 warps, for dγ then dβ
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n = a.n;
    float4 pw[VPL], pb[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) pw[i] = pb[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int r0 = blockIdx.x * LN_ROWS_V;
    for (int rr = warp; rr < LN_ROWS_V; rr += 8) {
        const int r = r0 + rr;
        if (r >= a.rows) break;
        const float* xr = a.x + static_cast<size_t>(a.gather ? a.gather[r] : r) * n + 4 * lane;
        const float* dyr = a.dy + static_cast<size_t>(r) * n + 4 * lane;
        const float mean = a.mean[r], rstd = a.rstd[r];
        float* dst = a.dx ? a.dx + static_cast<size_t>(a.scatter ? a.scatter[r] : r) * n + 4 * lane : nullptr;
        // the accumulated dx is read with the row's inputs, so the row waits on one round of loads
        const bool acc_in = dst && a.accumulate && !a.scatter;
        float4 prev[VPL];
#pragma unroll
        for (int i = 0; i < VPL; ++i) prev[i] = acc_in ? ld4(dst + 128 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 xh[VPL], g[VPL];
        float sg = 0.f, sgx = 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const float4 x = ld4(xr + 128 * i), dy = ld4(dyr + 128 * i), w = ld4(a.w + 4 * lane + 128 * i);
            xh[i] = make_float4((x.x - mean) * rstd, (x.y - mean) * rstd, (x.z - mean) * rstd, (x.w - mean) * rstd);
            g[i] = make_float4(dy.x * w.x, dy.y * w.y, dy.z * w.z, dy.w * w.w);
            sg += (g[i].x + g[i].y) + (g[i].z + g[i].w);
            sgx += (g[i].x * xh[i].x + g[i].y * xh[i].y) + (g[i].z * xh[i].z + g[i].w * xh[i].w);
            pw[i].x += dy.x * xh[i].x; pw[i].y += dy.y * xh[i].y; pw[i].z += dy.z * xh[i].z; pw[i].w += dy.w * xh[i].w;
            pb[i].x += dy.x; pb[i].y += dy.y; pb[i].z += dy.z; pb[i].w += dy.w;
        }
        const float mg = warp_sum(sg) / n, mgx = warp_sum(sgx) / n;
        if (dst) {
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                float4 d = make_float4(rstd * (g[i].x - mg - xh[i].x * mgx), rstd * (g[i].y - mg - xh[i].y * mgx),
                                       rstd * (g[i].z - mg - xh[i].z * mgx), rstd * (g[i].w - mg - xh[i].w * mgx));
                float* p = dst + 128 * i;
                if (a.scatter) {
                    atomicAdd(p, d.x); atomicAdd(p + 1, d.y); atomicAdd(p + 2, d.z); atomicAdd(p + 3, d.w);
                } else {
                    if (a.accumulate) {
                        d.x += prev[i].x; d.y += prev[i].y; d.z += prev[i].z; d.w += prev[i].w;
                    }
                    *reinterpret_cast<float4*>(p) = d;
                }
            }
        }
    }
    if (!a.dw && !a.db) return;
#pragma unroll
    for (int i = 0; i < VPL; ++i) *reinterpret_cast<float4*>(&red[warp][4 * lane + 128 * i]) = pw[i];
    __syncthreads();
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
        float sw = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sw += red[w][c];
        if (a.dw) atomicAdd(a.dw + c, sw);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < VPL; ++i) *reinterpret_cast<float4*>(&red[warp][4 * lane + 128 * i]) = pb[i];
    __syncthreads();
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
        float sb = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sb += red[w][c];
        if (a.db) atomicAdd(a.db + c, sb);
    }
}

// The persistent LayerNorm backward for n = 128·VPL: a warp per row, rows strided over a grid of
// LN_PART_CTAS_PER_SM CTAs of LNB_WARPS warps per SM, every load of a row (x, dy and the accumulated dx) issued
// before its reductions.
// dγ and dβ partials stay per (warp, lane, column) in shared memory (no atomics); at the end each CTA sums its warps
// in a fixed order into part[cta][2n], and ln_bwd_reduce_kernel adds the CTAs' partials to dγ and dβ in a fixed
// order — the same gradient bits on every run.
constexpr int LNB_WARPS = 16;
template <int VPL>
__global__ void __launch_bounds__(LNB_WARPS * 32, 1) ln_bwd_rows_kernel(LnBwd a) {
    extern __shared__ float4 lnp[];   // [LNB_WARPS][dγ | dβ][VPL][32 lanes] float4
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n = a.n;
    float4* pw = lnp + (warp * 2) * VPL * 32 + lane;
    float4* pb = pw + VPL * 32;
#pragma unroll
    for (int i = 0; i < VPL; ++i) pw[32 * i] = pb[32 * i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = blockIdx.x * LNB_WARPS + warp; r < a.rows; r += gridDim.x * LNB_WARPS) {
        const float* xr = a.x + static_cast<size_t>(a.gather ? a.gather[r] : r) * n + 4 * lane;
        const float* dyr = a.dy + static_cast<size_t>(r) * n + 4 * lane;
        float* dst = a.dx ? a.dx + static_cast<size_t>(a.scatter ? a.scatter[r] : r) * n + 4 * lane : nullptr;
        const bool acc_in = dst && a.accumulate && !a.scatter;
        float4 x[VPL], dy[VPL], prev[VPL];
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            x[i] = ld4(xr + 128 * i);
            dy[i] = ld4(dyr + 128 * i);
            prev[i] = acc_in ? ld4(dst + 128 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float mean = a.mean[r], rstd = a.rstd[r];
        float sg = 0.f, sgx = 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const float4 w = ld4(a.w + 4 * lane + 128 * i);
            float4 xh = make_float4((x[i].x - mean) * rstd, (x[i].y - mean) * rstd, (x[i].z - mean) * rstd,
                                    (x[i].w - mean) * rstd);
            float4 q = pw[32 * i], b = pb[32 * i];
            q.x += dy[i].x * xh.x; q.y += dy[i].y * xh.y; q.z += dy[i].z * xh.z; q.w += dy[i].w * xh.w;
            b.x += dy[i].x; b.y += dy[i].y; b.z += dy[i].z; b.w += dy[i].w;
            pw[32 * i] = q;
            pb[32 * i] = b;
            const float4 g = make_float4(dy[i].x * w.x, dy[i].y * w.y, dy[i].z * w.z, dy[i].w * w.w);
            sg += (g.x + g.y) + (g.z + g.w);
            sgx += (g.x * xh.x + g.y * xh.y) + (g.z * xh.z + g.w * xh.w);
            x[i] = xh;    // x̂ and g replace x and dy
            dy[i] = g;
        }
        const float mg = warp_sum(sg) / n, mgx = warp_sum(sgx) / n;
        if (!dst) continue;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            float4 d = make_float4(rstd * (dy[i].x - mg - x[i].x * mgx), rstd * (dy[i].y - mg - x[i].y * mgx),
                                   rstd * (dy[i].z - mg - x[i].z * mgx), rstd * (dy[i].w - mg - x[i].w * mgx));
            float* p = dst + 128 * i;
            if (a.scatter) {
                atomicAdd(p, d.x); atomicAdd(p + 1, d.y); atomicAdd(p + 2, d.z); atomicAdd(p + 3, d.w);
            } else {
                if (a.accumulate) { d.x += prev[i].x; d.y += prev[i].y; d.z += prev[i].z; d.w += prev[i].w; }
                *reinterpret_cast<float4*>(p) = d;
            }
        }
    }
    if (!a.dw && !a.db) return;
    __syncthreads();
    // column c = 128·i + 4·l + k lives in lane l's float4 i, component k; the 8 warps summed in order
    const float* lf = reinterpret_cast<const float*>(lnp);
    for (int c = threadIdx.x; c < 2 * n; c += blockDim.x) {
        const int which = c >= n, cc = c - which * n, i = cc >> 7, l = (cc & 127) >> 2, k = cc & 3;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < LNB_WARPS; ++w) sum += lf[(((w * 2 + which) * VPL + i) * 32 + l) * 4 + k];
        a.part[static_cast<size_t>(blockIdx.x) * 2 * n + c] = sum;
    }
}

// dγ += Σ_cta part[cta][c], dβ += Σ_cta part[cta][n + c] in a fixed order: a CTA takes 32 columns; its 32 warps sum
// the CTAs b ≡ warp (mod 32) in increasing b, then warp 0 adds the 32 sums in warp order.
__global__ void __launch_bounds__(1024) ln_bwd_reduce_kernel(const float* __restrict__ part, int ctas, int n, float* dw,
                                                            float* db) {
    __shared__ float red[32][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x * 32 + lane;
    float sum = 0.f;
    if (c < 2 * n) {
        int b = warp;
        for (; b + 96 < ctas; b += 128) {   // four loads in flight, summed in b order
            float s4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) s4[u] = part[static_cast<size_t>(b + 32 * u) * 2 * n + c];
#pragma unroll
            for (int u = 0; u < 4; ++u) sum += s4[u];
        }
        for (; b < ctas; b += 32) sum += part[static_cast<size_t>(b) * 2 * n + c];
    }
    red[warp][lane] = sum;
    __syncthreads();
    if (warp == 0 && c < 2 * n) {
        float t = 0.f;
        for (int w = 0; w < 32; ++w) t += red[w][lane];
        float* dst = c < n ? dw : db;
        if (dst) dst[c < n ? c : c - n] += t;
    }
}

// ------------------------------------------------------------------------------------------------ GeGLU
DEVI float ld_f(const float* p) { return *p; }
DEVI float ld_f(const __nv_bfloat16* p) { return bf(*p); }
DEVI void st_split(__nv_bfloat16* hi, __nv_bfloat16* lo, size_t i, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    if (lo) lo[i] = __float2bfloat16_rn(v - bf(h));
}

// Four consecutive elements per thread: 16-byte fp32 and 8-byte bf16 accesses (callers guarantee 4-element alignment).
struct F4 { float v[4]; };
DEVI F4 ldv4(const float* p) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    return F4{{x.x, x.y, x.z, x.w}};
}
DEVI F4 ldv4(const __nv_bfloat16* p) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&x.x), b = *reinterpret_cast<const __nv_bfloat162*>(&x.y);
    return F4{{__low2float(a), __high2float(a), __low2float(b), __high2float(b)}};
}
DEVI void st4(__nv_bfloat16* p, const F4& f) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(f.v[0], f.v[1]), b = __floats2bfloat162_rn(f.v[2], f.v[3]);
    uint2 x;
    x.x = *reinterpret_cast<const uint32_t*>(&a);
    x.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = x;
}
DEVI void st4_split(__nv_bfloat16* hi, __nv_bfloat16* lo, size_t i, const F4& f) {
    F4 h, l;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        h.v[k] = bf(__float2bfloat16_rn(f.v[k]));
        l.v[k] = f.v[k] - h.v[k];
    }
    st4(hi + i, h);   // h holds bf16 values: rounding them again is exact
    if (lo) st4(lo + i, l);
}

// act = gelu(u) · gate, [u | gate] = wide row (bf16, or fp32 in the accurate forward with act's low part).
// Thread = 4 consecutive columns of one row (I a multiple of 4).
template <typename Src>
__global__ void geglu_fwd_kernel(const Src* __restrict__ wide, int rows, int I, __nv_bfloat16* __restrict__ act,
                                 __nv_bfloat16* __restrict__ act_lo) {
    const unsigned I4 = static_cast<unsigned>(I) >> 2;
    const unsigned j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= static_cast<unsigned>(rows) * I4) return;
    const unsigned r = j / I4, c = (j - r * I4) * 4;
    const Src* row = wide + static_cast<size_t>(r) * 2 * I;
    const F4 u = ldv4(row + c), g = ldv4(row + I + c);
    F4 o;
#pragma unroll
    for (int k = 0; k < 4; ++k) o.v[k] = gelu_exact(u.v[k]) * g.v[k];
    st4_split(act, act_lo, static_cast<size_t>(r) * I + c, o);
}
// dgate = dy·gelu(u); du = dy·gate·gelu'(u)
template <typename Src>
__global__ void geglu_bwd_kernel(const Src* __restrict__ wide, const float* __restrict__ dact, int rows, int I,
                                 __nv_bfloat16* __restrict__ dwide) {
    const unsigned I4 = static_cast<unsigned>(I) >> 2;
    const unsigned j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= static_cast<unsigned>(rows) * I4) return;
    const unsigned r = j / I4, c = (j - r * I4) * 4;
    const Src* row = wide + static_cast<size_t>(r) * 2 * I;
    const F4 u = ldv4(row + c), g = ldv4(row + I + c), dy = ldv4(dact + static_cast<size_t>(r) * I + c);
    F4 dg, du;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        dg.v[k] = dy.v[k] * gelu_exact(u.v[k]);
        du.v[k] = dy.v[k] * g.v[k] * gelu_grad(u.v[k]);
    }
    __nv_bfloat16* out = dwide + static_cast<size_t>(r) * 2 * I;
    st4(out + I + c, dg);
    st4(out + c, du);
}

// ------------------------------------------------------------------------------------------------ masked elementwise
// Elementwise kernels: thread = 4 consecutive elements (4-element aligned buffers; a ragged tail element by element).
// y32 = a32 + mask(b32)   (a residual branch with dropout, HeadLayerForward)
__global__ void add_masked_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y, size_t n,
                                  Mask m) {
    const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= n) return;
    if (i + 4 > n) {   // the ragged tail
        for (size_t k = i; k < n; ++k) y[k] = a[k] + b[k] * dmask(m, k);
        return;
    }
    const F4 x = ldv4(a + i), z = ldv4(b + i);
    float4 o;
    o.x = x.v[0] + z.v[0] * dmask(m, i);
    o.y = x.v[1] + z.v[1] * dmask(m, i + 1);
    o.z = x.v[2] + z.v[2] * dmask(m, i + 2);
    o.w = x.v[3] + z.v[3] * dmask(m, i + 3);
    *reinterpret_cast<float4*>(y + i) = o;
}
// act = mask(relu(pre))   (linear1 → ReLU → dropout, HeadLayerForward); pre bf16 or fp32 (+ act's low part)
template <typename Src>
__global__ void relu_mask_kernel(const Src* __restrict__ pre, __nv_bfloat16* __restrict__ act,
                                 __nv_bfloat16* __restrict__ act_lo, size_t n, Mask m) {
    const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= n) return;
    if (i + 4 > n) {
        for (size_t k = i; k < n; ++k) st_split(act, act_lo, k, fmaxf(ld_f(pre + k), 0.f) * dmask(m, k));
        return;
    }
    F4 x = ldv4(pre + i);
#pragma unroll
    for (int k = 0; k < 4; ++k) x.v[k] = fmaxf(x.v[k], 0.f) * dmask(m, i + k);
    st4_split(act, act_lo, i, x);
}
// dx16 = bf16(mask(d32) · [pre > 0])
template <typename Src>
__global__ void relu_mask_bwd_kernel(const float* __restrict__ d, const Src* __restrict__ pre,
                                     __nv_bfloat16* __restrict__ dx, size_t n, Mask m) {
    const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= n) return;
    if (i + 4 > n) {
        for (size_t k = i; k < n; ++k) dx[k] = __float2bfloat16_rn(ld_f(pre + k) > 0.f ? d[k] * dmask(m, k) : 0.f);
        return;
    }
    const F4 p = ldv4(pre + i);
    F4 g = ldv4(d + i);
#pragma unroll
    for (int k = 0; k < 4; ++k) g.v[k] = p.v[k] > 0.f ? g.v[k] * dmask(m, i + k) : 0.f;
    st4(dx + i, g);
}
// y16 = bf16(mask(x32))
__global__ void cast_mask_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, size_t n, Mask m) {
    const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= n) return;
    if (i + 4 > n) {
        for (size_t k = i; k < n; ++k) y[k] = __float2bfloat16_rn(x[k] * dmask(m, k));
        return;
    }
    F4 v = ldv4(x + i);
#pragma unroll
    for (int k = 0; k < 4; ++k) v.v[k] = v.v[k] * dmask(m, i + k);
    st4(y + i, v);
}

// db[c] += Σ_r d[r, c]  (d fp32 or bf16); a CTA takes 64 rows × 256 columns
template <typename T>
__global__ void colsum_kernel(const T* __restrict__ d, int rows, int n, float* __restrict__ db) {
    const int c = blockIdx.y * blockDim.x + threadIdx.x;
    if (c >= n) return;
    const int r0 = blockIdx.x * 64, r1 = min(rows, r0 + 64);
    float s = 0.f;
    for (int r = r0; r < r1; ++r) {
        if constexpr (sizeof(T) == 4) s += d[static_cast<size_t>(r) * n + c];
        else s += bf(d[static_cast<size_t>(r) * n + c]);
    }
    atomicAdd(db + c, s);
}

// db[c] += Σ_r d[r, c] for bf16 d with n a multiple of 8: a CTA takes 256 rows × 256 columns, thread (row lane rl,
// column group cg) summing 8 columns of rows rl, rl + 8, … with one 16-byte load per row; the 8 row lanes then meet in
// shared memory.
constexpr int CS_ROWS = 256;
__global__ void __launch_bounds__(256) colsum8_kernel(const __nv_bfloat16* __restrict__ d, int rows, int n,
                                                      float* __restrict__ db) {
    __shared__ float part[8][256];
    const int cg = threadIdx.x & 31, rl = threadIdx.x >> 5;
    const int c0 = blockIdx.y * 256 + cg * 8;
    const int r0 = blockIdx.x * CS_ROWS, r1 = min(rows, r0 + CS_ROWS);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (c0 < n) {
        for (int r = r0 + rl; r < r1; r += 8) {
            const uint4 x = *reinterpret_cast<const uint4*>(d + static_cast<size_t>(r) * n + c0);
            const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 u = __bfloat1622float2(xa[k]);
                acc[2 * k] += u.x;
                acc[2 * k + 1] += u.y;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) part[rl][cg * 8 + k] = acc[k];
    __syncthreads();
    const int c = blockIdx.y * 256 + threadIdx.x;
    if (c < n) {
        float sum = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) sum += part[q][threadIdx.x];
        atomicAdd(db + c, sum);
    }
}

// grad[ids[t]] += d[t]   (embedding rows)
__global__ void scatter_rows_kernel(const float* __restrict__ d, const int32_t* __restrict__ ids, int rows, int n,
                                    float* __restrict__ grad) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(rows) * n) return;
    const size_t r = i / n, c = i % n;
    atomicAdd(grad + static_cast<size_t>(ids[r]) * n + c, d[i]);
}
// gtype[qtype[item(t)]] += d[t]: 3 type rows accumulated in shared memory per 64 rows
__global__ void type_grad_kernel(const float* __restrict__ d, const int32_t* __restrict__ tok_item,
                                 const int32_t* __restrict__ qtype, int rows, int n, float* __restrict__ grad) {
    extern __shared__ float acc[];   // [3][n]
    for (int i = threadIdx.x; i < 3 * n; i += blockDim.x) acc[i] = 0.f;
    __syncthreads();
    const int r0 = blockIdx.x * 64, r1 = min(rows, r0 + 64);
    for (int r = r0; r < r1; ++r) {
        const int t = qtype[tok_item[r]];
        for (int c = threadIdx.x; c < n; c += blockDim.x) acc[t * n + c] += d[static_cast<size_t>(r) * n + c];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 3 * n; i += blockDim.x)
        if (acc[i] != 0.f) atomicAdd(grad + i, acc[i]);
}

// ------------------------------------------------------------------------------------------------ scorer
// pre32 [M, n] (Linear1 + bias) → act = gelu(pre) (bf16 for the dW product of Linear2 is not needed: Linear2 is a
// dot); logits[m] = Σ act·w2 + b2.  One warp per marker.
__global__ void scorer_out_kernel(const float* __restrict__ pre, int M, int n, const float* __restrict__ w2,
                                  const float* __restrict__ b2, float* __restrict__ logits) {
    const int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (m >= M) return;
    float s = 0.f;
    for (int c = lane; c < n; c += 32) s += gelu_exact(pre[static_cast<size_t>(m) * n + c]) * w2[c];
    s = warp_sum(s);
    if (lane == 0) logits[m] = s + b2[0];
}
// dpre[m, c] = dlogit[m] · w2[c] · gelu'(pre[m, c]) → bf16 for the dX / dW products, and in fp32 summed into db1;
// dw2[c] += Σ_m dlogit[m] · gelu(pre[m, c]); db2 += Σ_m dlogit[m]   (Ops.LinearBackward + Ops.GeluBackward).
__global__ void scorer_bwd_kernel(const float* __restrict__ pre, const float* __restrict__ dlogit, int M, int n,
                                  const float* __restrict__ w2, __nv_bfloat16* __restrict__ dpre, float* __restrict__ db1,
                                  float* __restrict__ dw2, float* __restrict__ db2) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < n) {
        float acc = 0.f, acc1 = 0.f;
        for (int m = 0; m < M; ++m) {
            const float p = pre[static_cast<size_t>(m) * n + c];
            acc += dlogit[m] * gelu_exact(p);
            const float d = dlogit[m] * w2[c] * gelu_grad(p);
            acc1 += d;
            dpre[static_cast<size_t>(m) * n + c] = __float2bfloat16_rn(d);
        }
        if (dw2) atomicAdd(dw2 + c, acc);
        if (db1) atomicAdd(db1 + c, acc1);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && db2) {
        float s = 0.f;
        for (int m = 0; m < M; ++m) s += dlogit[m];
        atomicAdd(db2, s);
    }
}

// ------------------------------------------------------------------------------------------------ optimizer
// Σ g² over [0, n) in double, per CTA partials reduced with atomics (Gradients.ClipByGlobalNorm sums in double).
__global__ void __launch_bounds__(256) sumsq_kernel(const float* __restrict__ g, size_t n, double* __restrict__ out) {
    // four independent fp64 accumulators over 16-byte loads keep enough loads in flight to stream at HBM rate
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    const size_t n4 = reinterpret_cast<uintptr_t>(g) & 15 ? 0 : n / 4;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = g4[i];
        s0 = fma(static_cast<double>(v.x), static_cast<double>(v.x), s0);
        s1 = fma(static_cast<double>(v.y), static_cast<double>(v.y), s1);
        s2 = fma(static_cast<double>(v.z), static_cast<double>(v.z), s2);
        s3 = fma(static_cast<double>(v.w), static_cast<double>(v.w), s3);
    }
    for (size_t i = 4 * n4 + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        s0 = fma(static_cast<double>(g[i]), static_cast<double>(g[i]), s0);
    double s = (s0 + s1) + (s2 + s3);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double ws[32];
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += ws[w];
        out[blockIdx.x] = t;   // one partial per block: the sum order does not depend on scheduling
    }
}

// AdamW.Step for one contiguous parameter range: g = grad · gscale (the clipping factor and the 1/world average folded
// in), decoupled decay, bias-corrected moments, then the bf16 shadow the products read.
__global__ void adamw_kernel(AdamArgs a) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= a.n) return;
    const float gsc = a.gscale ? static_cast<float>(*a.gscale) : 1.0f;
    const float g = __fmul_rn(a.grad[i], gsc);
    float p = __fmul_rn(a.param[i], a.decay);
    const float m = __fadd_rn(__fmul_rn(a.b1, a.m[i]), __fmul_rn(1.0f - a.b1, g));
    const float v = __fadd_rn(__fmul_rn(a.b2, a.v[i]), __fmul_rn(__fmul_rn(1.0f - a.b2, g), g));
    const float den = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), a.sqrt_c2), a.eps);
    p = __fsub_rn(p, __fdiv_rn(__fmul_rn(a.step_size, m), den));
    a.param[i] = p;
    a.m[i] = m;
    a.v[i] = v;
    if (a.shadow) st_split(a.shadow, a.shadow_lo, i, p);
}

// Gradients.ClipByGlobalNorm on the rank average g_sum / world: norm = sqrt(Σ g_sum²) / world,
// coef = max_norm / (norm + 1e-6); the factor applied to g_sum is min(1, coef) / world (world = 1: the reference's).
// One CTA of 256 threads: the SUMSQ_BLOCKS partials summed in a fixed order (strided per thread, then a fixed tree).
__global__ void __launch_bounds__(256) clip_scale_kernel(const double* partials, double max_norm, int world,
                                                         double* sumsq, double* scale, double* norm_out) {
    double s = 0.0;
    for (int i = threadIdx.x; i < SUMSQ_BLOCKS; i += blockDim.x) s += partials[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double ws[8];
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x != 0) return;
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += ws[w];
    *sumsq = t;
    const double norm = sqrt(t) / world;
    const double coef = max_norm / (norm + 1e-6);
    *scale = (coef < 1.0 ? coef : 1.0) / world;
    if (norm_out) *norm_out = norm;
}

// ------------------------------------------------------------------------------------------------ objective
// RlcdObjective.Compute with supplied standard-normal draws (RlcdObjective.cs:57-155) and Calibration.ProperReward
// (Calibration.cs:76-119, every option unmasked), one CTA: (group, item) samples in parallel, then the advantage
// normalisation and every running sum on one thread in the reference's order, so the result does not depend on the
// launch shape.  Softmax is fp32 as SimdOps.Softmax (SimdOps.cs:275-291); everything else fp64.
DEVI void softmax_f32(float* v, int k) {
    float mx = -INFINITY;
    for (int o = 0; o < k; ++o) mx = fmaxf(mx, v[o]);
    if (mx == -INFINITY) { for (int o = 0; o < k; ++o) v[o] = 0.f; return; }
    float total = 0.f;
    for (int o = 0; o < k; ++o) { const float e = expf(v[o] - mx); v[o] = e; total = __fadd_rn(total, e); }
    const float sc = total > 0.f ? 1.0f / total : 0.f;
    for (int o = 0; o < k; ++o) v[o] = __fmul_rn(v[o], sc);
}

__global__ void __launch_bounds__(256) rlcd_kernel(RlcdArgs a) {
    const int n = a.n_items, G = a.groups, M = a.M;
    double* eps = a.scratch;                  // [G][M]
    double* reward = eps + static_cast<size_t>(G) * M;   // [G][n]
    double* adv = reward + static_cast<size_t>(G) * n;   // [G][n]
    float* q = reinterpret_cast<float*>(adv + static_cast<size_t>(G) * n);   // [G][M] perturbed, then [M] clean
    for (int p = threadIdx.x; p < G * n; p += blockDim.x) {
        const int g = p / n, i = p % n;
        const int k = a.mk_count[i], o0 = a.mk_start[i];
        double* e = eps + static_cast<size_t>(g) * M + o0;
        float* qq = q + static_cast<size_t>(g) * M + o0;
        double mean = 0.0;
        for (int o = 0; o < k; ++o) { e[o] = a.draws[static_cast<size_t>(g) * M + o0 + o] * a.sigma; mean += e[o]; }
        mean /= k;
        for (int o = 0; o < k; ++o) e[o] -= mean;
        for (int o = 0; o < k; ++o) qq[o] = __double2float_rn(static_cast<double>(a.logits[o0 + o]) + e[o]);
        softmax_f32(qq, k);
        const float* t = a.targets + o0;
        double logs = 0.0, dot = 0.0, nsq = 0.0;
        for (int o = 0; o < k; ++o) {
            const double qo = qq[o];
            logs += t[o] * fmax(log(fmax(qo, 1e-12)), -9.21);
            dot += t[o] * qo;
            nsq += qo * qo;
        }
        double r = logs + a.w_sph * (dot / fmax(sqrt(nsq), 1e-9));
        if (a.qtype[i] == 1) {   // QuestionType.Score: ranked probability score
            const int kk = k > 2 ? k : 2;
            double cq = 0.0, ct = 0.0, rps = 0.0;
            for (int o = 0; o < k; ++o) { cq += qq[o]; ct += t[o]; rps += (cq - ct) * (cq - ct); }
            r -= a.w_rps * rps / (kk - 1);
        }
        reward[static_cast<size_t>(g) * n + i] = r;
    }
    __syncthreads();
    const int count = G * n;
    if (threadIdx.x == 0) {
        double total = 0.0;
        for (int i = 0; i < n; ++i) {
            double mean = 0.0;
            for (int g = 0; g < G; ++g) mean += reward[static_cast<size_t>(g) * n + i];
            mean /= G;
            for (int g = 0; g < G; ++g) {
                adv[static_cast<size_t>(g) * n + i] = reward[static_cast<size_t>(g) * n + i] - mean;
                total += adv[static_cast<size_t>(g) * n + i];
            }
        }
        const double gm = total / count;
        double var = 0.0;
        for (int g = 0; g < G; ++g)
            for (int i = 0; i < n; ++i) {
                const double d = adv[static_cast<size_t>(g) * n + i] - gm;
                var += d * d;
            }
        const double sd = count > 1 ? sqrt(var / (count - 1)) : 0.0;
        for (int j = 0; j < count; ++j) adv[j] /= sd + 1e-6;
    }
    __syncthreads();
    // per item: policy-gradient term + soft cross-entropy gradient
    float* pc = q;   // the clean softmax reuses group 0's slots
    const double s2 = a.sigma * a.sigma;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int k = a.mk_count[i], o0 = a.mk_start[i];
        for (int o = 0; o < k; ++o) pc[o0 + o] = a.logits[o0 + o];
        softmax_f32(pc + o0, k);
        const float* t = a.targets + o0;
        double mass = 0.0;
        for (int o = 0; o < k; ++o) mass += t[o];
        for (int o = 0; o < k; ++o) {
            double gr = 0.0;
            for (int g = 0; g < G; ++g)
                gr -= adv[static_cast<size_t>(g) * n + i] * eps[static_cast<size_t>(g) * M + o0 + o] / s2 / count;
            gr += a.w_ce * (static_cast<double>(pc[o0 + o]) * mass - t[o]) / n;
            a.dlogits[o0 + o] = __double2float_rn(gr * a.scale);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double policy = 0.0, ce = 0.0, rsum = 0.0;
        for (int i = 0; i < n; ++i) {
            const int k = a.mk_count[i], o0 = a.mk_start[i];
            for (int g = 0; g < G; ++g) {
                double logp = 0.0;
                for (int o = 0; o < k; ++o) {
                    const double e = eps[static_cast<size_t>(g) * M + o0 + o];
                    logp -= e * e / (2 * s2);
                }
                policy -= adv[static_cast<size_t>(g) * n + i] * logp / count;
                rsum += reward[static_cast<size_t>(g) * n + i];
            }
            for (int o = 0; o < k; ++o) ce -= a.targets[o0 + o] * log(fmax(static_cast<double>(pc[o0 + o]), 1e-30)) / n;
        }
        a.result[0] = policy + a.w_ce * ce;
        a.result[1] = policy;
        a.result[2] = ce;
        a.result[3] = rsum / count;
    }
}

// Eight elements per thread: two 16-byte loads, one 16-byte store.
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, size_t n) {
    const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i + 8 <= n) {
        const float4 a = *reinterpret_cast<const float4*>(x + i), b = *reinterpret_cast<const float4*>(x + i + 4);
        const __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(a.z, a.w),
                             h2 = __floats2bfloat162_rn(b.x, b.y), h3 = __floats2bfloat162_rn(b.z, b.w);
        *reinterpret_cast<uint4*>(y + i) =
            make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                       *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
    } else {
        for (size_t k = i; k < n; ++k) y[k] = __float2bfloat16_rn(x[k]);
    }
}
__global__ void f32_split_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo,
                                 size_t n) {
    const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i + 4 <= n) st4_split(hi, lo, i, ldv4(x + i));
    else for (size_t k = i; k < n; ++k) st_split(hi, lo, k, x[k]);
}

}  // namespace tr

// ------------------------------------------------------------------------------------------------ launchers
static unsigned blocks_for(size_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

int ln_fwd(const tr::LnFwd& a, cudaStream_t s) {
    if (a.rows <= 0) return OK;
    const unsigned g = blocks_for(static_cast<size_t>(a.rows) * 32, 256);
    switch (a.n % 128 == 0 ? a.n / 128 : 0) {
        case 1: tr::ln_fwd_vec_kernel<1><<<g, 256, 0, s>>>(a); break;
        case 2: tr::ln_fwd_vec_kernel<2><<<g, 256, 0, s>>>(a); break;
        case 4: tr::ln_fwd_vec_kernel<4><<<g, 256, 0, s>>>(a); break;
        case 6: tr::ln_fwd_vec_kernel<6><<<g, 256, 0, s>>>(a); break;
        case 8: tr::ln_fwd_vec_kernel<8><<<g, 256, 0, s>>>(a); break;
        default:
            if (a.n <= 128) tr::ln_fwd_kernel<4><<<g, 256, 0, s>>>(a);
            else if (a.n <= 256) tr::ln_fwd_kernel<8><<<g, 256, 0, s>>>(a);
            else if (a.n <= 768) tr::ln_fwd_kernel<24><<<g, 256, 0, s>>>(a);
            else if (a.n <= 1024) tr::ln_fwd_kernel<32><<<g, 256, 0, s>>>(a);
            else { set_error("LayerNorm width above 1024"); return ERR_NOT_SUPPORTED; }
    }
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

template <int VPL>
static int ln_bwd_rows(const tr::LnBwd& a, cudaStream_t s) {
    constexpr int smem = tr::LNB_WARPS * 2 * VPL * 32 * 16;
    static DeviceOnce attr;
    int dev = 0, nsm = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(tr::ln_bwd_rows_kernel<VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr.mark(dev);
    }
    if (int e = sm_count(dev, &nsm)) return e;
    const int want = (a.rows + tr::LNB_WARPS - 1) / tr::LNB_WARPS, cap = tr::LN_PART_CTAS_PER_SM * nsm;
    const int ctas = want < cap ? want : cap;
    tr::ln_bwd_rows_kernel<VPL><<<ctas, tr::LNB_WARPS * 32, smem, s>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    if (a.dw || a.db) {
        tr::ln_bwd_reduce_kernel<<<blocks_for(2 * static_cast<size_t>(a.n), 32), 1024, 0, s>>>(a.part, ctas, a.n, a.dw, a.db);
        count_launch();
        LAYA_CUDA(cudaGetLastError());
    }
    return OK;
}

int ln_bwd(const tr::LnBwd& a, cudaStream_t s) {
    if (a.rows <= 0) return OK;
    if (a.part && a.n % 128 == 0) {   // the persistent form (widths 768 and 1024: ModernBERT-base and -large)
        switch (a.n / 128) {
            case 6: return ln_bwd_rows<6>(a, s);
            case 8: return ln_bwd_rows<8>(a, s);
            default: break;
        }
    }
    if (a.n % 128 == 0 && a.n <= 1024 && a.n != 384 && a.n != 640 && a.n != 896) {
        const unsigned g = blocks_for(static_cast<size_t>(a.rows), tr::LN_ROWS_V);
        switch (a.n / 128) {
            case 1: tr::ln_bwd_vec_kernel<1><<<g, 256, 0, s>>>(a); break;
            case 2: tr::ln_bwd_vec_kernel<2><<<g, 256, 0, s>>>(a); break;
            case 4: tr::ln_bwd_vec_kernel<4><<<g, 256, 0, s>>>(a); break;
            case 6: tr::ln_bwd_vec_kernel<6><<<g, 256, 0, s>>>(a); break;
            case 8: tr::ln_bwd_vec_kernel<8><<<g, 256, 0, s>>>(a); break;
        }
    } else {
        const unsigned g = blocks_for(static_cast<size_t>(a.rows), tr::LN_ROWS);
        if (a.n <= 128) tr::ln_bwd_kernel<4><<<g, 256, 0, s>>>(a);
        else if (a.n <= 256) tr::ln_bwd_kernel<8><<<g, 256, 0, s>>>(a);
        else if (a.n <= 768) tr::ln_bwd_kernel<24><<<g, 256, 0, s>>>(a);
        else if (a.n <= 1024) tr::ln_bwd_kernel<32><<<g, 256, 0, s>>>(a);
        else { set_error("LayerNorm width above 1024"); return ERR_NOT_SUPPORTED; }
    }
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

#define LAUNCH1(kern, n, ...)                                                           \
    do {                                                                                \
        if ((n) > 0) {                                                                  \
            tr::kern<<<blocks_for((n), 256), 256, 0, s>>>(__VA_ARGS__);                 \
            count_launch();                                                             \
            LAYA_CUDA(cudaGetLastError());                                              \
        }                                                                               \
        return OK;                                                                      \
    } while (0)

// The 4-wide kernels need 4-element-aligned addresses (and, for GeGLU, rows of a multiple of 4 columns).
static bool aligned4(size_t n, std::initializer_list<const void*> ptrs, size_t elem_bytes_min = 2) {
    (void)n;
    for (const void* p : ptrs)
        if (p && (reinterpret_cast<uintptr_t>(p) % (4 * elem_bytes_min))) return false;
    return true;
}
#define LAUNCH4(kern, n, ...)                                                           \
    do {                                                                                \
        if ((n) > 0) {                                                                  \
            tr::kern<<<blocks_for(((n) + 3) / 4, 256), 256, 0, s>>>(__VA_ARGS__);       \
            count_launch();                                                             \
            LAYA_CUDA(cudaGetLastError());                                              \
        }                                                                               \
        return OK;                                                                      \
    } while (0)
#define REQUIRE4(n, ...)                                                                                        \
    do {                                                                                                        \
        if (!aligned4((n), {__VA_ARGS__})) {                                                                    \
            set_error("elementwise kernel: buffers must be 4-element aligned");                                 \
            return ERR_ARGUMENT;                                                                                \
        }                                                                                                       \
    } while (0)

static int geglu_width(int I) {
    if (I % 4) { set_error("GeGLU width must be a multiple of 4"); return ERR_ARGUMENT; }
    return OK;
}
int geglu_fwd(const __nv_bfloat16* wide, int rows, int I, __nv_bfloat16* act, cudaStream_t s) {
    if (geglu_width(I) != OK) return ERR_ARGUMENT;
    REQUIRE4(static_cast<size_t>(I), wide, act);
    LAUNCH4(geglu_fwd_kernel<__nv_bfloat16>, static_cast<size_t>(rows) * I, wide, rows, I, act, nullptr);
}
int geglu_fwd_f32(const float* wide, int rows, int I, __nv_bfloat16* act, __nv_bfloat16* act_lo, cudaStream_t s) {
    if (geglu_width(I) != OK) return ERR_ARGUMENT;
    REQUIRE4(static_cast<size_t>(I), wide, act, act_lo);
    LAUNCH4(geglu_fwd_kernel<float>, static_cast<size_t>(rows) * I, wide, rows, I, act, act_lo);
}
int geglu_bwd(const __nv_bfloat16* wide, const float* dact, int rows, int I, __nv_bfloat16* dwide, cudaStream_t s) {
    if (geglu_width(I) != OK) return ERR_ARGUMENT;
    REQUIRE4(static_cast<size_t>(I), wide, dact, dwide);
    LAUNCH4(geglu_bwd_kernel<__nv_bfloat16>, static_cast<size_t>(rows) * I, wide, dact, rows, I, dwide);
}
int geglu_bwd_f32(const float* wide, const float* dact, int rows, int I, __nv_bfloat16* dwide, cudaStream_t s) {
    if (geglu_width(I) != OK) return ERR_ARGUMENT;
    REQUIRE4(static_cast<size_t>(I), wide, dact, dwide);
    LAUNCH4(geglu_bwd_kernel<float>, static_cast<size_t>(rows) * I, wide, dact, rows, I, dwide);
}
int add_masked(const float* a, const float* b, float* y, size_t n, tr::Mask m, cudaStream_t s) {
    REQUIRE4(n, a, b, y);
    LAUNCH4(add_masked_kernel, n, a, b, y, n, m);
}
int relu_mask(const __nv_bfloat16* pre, __nv_bfloat16* act, size_t n, tr::Mask m, cudaStream_t s) {
    REQUIRE4(n, pre, act);
    LAUNCH4(relu_mask_kernel<__nv_bfloat16>, n, pre, act, nullptr, n, m);
}
int relu_mask_f32(const float* pre, __nv_bfloat16* act, __nv_bfloat16* act_lo, size_t n, tr::Mask m, cudaStream_t s) {
    REQUIRE4(n, pre, act, act_lo);
    LAUNCH4(relu_mask_kernel<float>, n, pre, act, act_lo, n, m);
}
int relu_mask_bwd(const float* d, const __nv_bfloat16* pre, __nv_bfloat16* dx, size_t n, tr::Mask m, cudaStream_t s) {
    REQUIRE4(n, d, pre, dx);
    LAUNCH4(relu_mask_bwd_kernel<__nv_bfloat16>, n, d, pre, dx, n, m);
}
int relu_mask_bwd_f32(const float* d, const float* pre, __nv_bfloat16* dx, size_t n, tr::Mask m, cudaStream_t s) {
    REQUIRE4(n, d, pre, dx);
    LAUNCH4(relu_mask_bwd_kernel<float>, n, d, pre, dx, n, m);
}
int cast_mask(const float* x, __nv_bfloat16* y, size_t n, tr::Mask m, cudaStream_t s) {
    REQUIRE4(n, x, y);
    LAUNCH4(cast_mask_kernel, n, x, y, n, m);
}
int f32_to_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s) {
    if (n == 0) return OK;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15)) {
        set_error("f32_to_bf16: buffers must be 16-byte aligned");
        return ERR_ARGUMENT;
    }
    tr::f32_to_bf16_kernel<<<blocks_for((n + 7) / 8, 256), 256, 0, s>>>(x, y, n);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int f32_split_bf16(const float* x, __nv_bfloat16* hi, __nv_bfloat16* lo, size_t n, cudaStream_t s) {
    REQUIRE4(n, x, hi, lo);
    LAUNCH4(f32_split_kernel, n, x, hi, lo, n);
}
int scatter_rows(const float* d, const int32_t* ids, int rows, int n, float* grad, cudaStream_t s) {
    LAUNCH1(scatter_rows_kernel, static_cast<size_t>(rows) * n, d, ids, rows, n, grad);
}

int colsum_f32(const float* d, int rows, int n, float* db, cudaStream_t s) {
    if (rows <= 0 || n <= 0) return OK;
    dim3 grid((rows + 63) / 64, (n + 255) / 256);
    tr::colsum_kernel<float><<<grid, 256, 0, s>>>(d, rows, n, db);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int colsum_bf16(const __nv_bfloat16* d, int rows, int n, float* db, cudaStream_t s) {
    if (rows <= 0 || n <= 0) return OK;
    if (n % 8 == 0 && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
        tr::colsum8_kernel<<<dim3((rows + tr::CS_ROWS - 1) / tr::CS_ROWS, (n + 255) / 256), 256, 0, s>>>(d, rows, n, db);
        count_launch();
        LAYA_CUDA(cudaGetLastError());
        return OK;
    }
    dim3 grid((rows + 63) / 64, (n + 255) / 256);
    tr::colsum_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(d, rows, n, db);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int type_grad(const float* d, const int32_t* tok_item, const int32_t* qtype, int rows, int n, float* grad, cudaStream_t s) {
    if (rows <= 0) return OK;
    tr::type_grad_kernel<<<(rows + 63) / 64, 256, sizeof(float) * 3 * n, s>>>(d, tok_item, qtype, rows, n, grad);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int scorer_out(const float* pre, int M, int n, const float* w2, const float* b2, float* logits, cudaStream_t s) {
    if (M <= 0) return OK;
    tr::scorer_out_kernel<<<blocks_for(static_cast<size_t>(M) * 32, 256), 256, 0, s>>>(pre, M, n, w2, b2, logits);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int scorer_bwd(const float* pre, const float* dlogit, int M, int n, const float* w2, __nv_bfloat16* dpre, float* db1,
               float* dw2, float* db2, cudaStream_t s) {
    if (M <= 0) return OK;
    tr::scorer_bwd_kernel<<<blocks_for(static_cast<size_t>(n), 256), 256, 0, s>>>(pre, dlogit, M, n, w2, dpre, db1, dw2, db2);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
size_t rlcd_scratch_bytes(int groups, int n_items, int M) {
    return sizeof(double) * (static_cast<size_t>(groups) * M + 2 * static_cast<size_t>(groups) * n_items) +
           sizeof(float) * static_cast<size_t>(groups > 0 ? groups : 1) * M;
}
int rlcd(const tr::RlcdArgs& a, cudaStream_t s) {
    if (a.n_items <= 0) return OK;
    tr::rlcd_kernel<<<1, 256, 0, s>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int sumsq(const float* g, size_t n, double* partials, cudaStream_t s) {
    if (n == 0) {
        LAYA_CUDA(cudaMemsetAsync(partials, 0, sizeof(double) * SUMSQ_BLOCKS, s));
        return OK;
    }
    tr::sumsq_kernel<<<SUMSQ_BLOCKS, 256, 0, s>>>(g, n, partials);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int clip_scale(const double* partials, double max_norm, int world, double* sumsq, double* scale, double* norm_out,
               cudaStream_t s) {
    tr::clip_scale_kernel<<<1, 256, 0, s>>>(partials, max_norm, world, sumsq, scale, norm_out);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}
int adamw(const tr::AdamArgs& a, cudaStream_t s) {
    if (a.n == 0) return OK;
    tr::adamw_kernel<<<blocks_for(a.n, 256), 256, 0, s>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace laya
