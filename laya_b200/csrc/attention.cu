// attention.cu — multi-head attention per question (segment), fused with what surrounds it.
//
// Replaces ModernBertEncoder.Attention (Laya/Models/ModernBertEncoder.cs:230-302) with its RopeCache
// (:341-401) and AttentionKernels.Scores/WeightedSum (Base/Numerics/AttentionKernels.cs:30-125), and
// DecisionModel.HeadAttention (Laya/Models/DecisionModel.cs:319-368, no rotary, no window).
//
//   * sequences are concatenated; a token attends only inside its own segment, positions restart at 0;
//   * sliding layers see keys [i - W, i + W] (inclusive), global layers the whole segment;
//   * rotary ("rotate half", RopeCache.Apply) is applied while Q and K tiles are loaded;
//   * softmax(q·kᵀ / √d) · V runs flash-style: 64-query tiles × 64-key tiles, online softmax in fp32;
//     keys outside [first window key, last window key] of the query tile are never loaded;
//   * the context rows come out as Q8_0 codes + block scales, ready for the Wo product
//     (PackedMatrixQ8_0.Multiply quantizes its input first, PackedMatrixQ8_0.cs:239).
// Q, K, V and P are fp16 on the tensor cores (mma.sync m16n8k16, fp32 accumulation); the reference is fp32,
// so this stage is compared within a tolerance.
#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace laya {
namespace attn {

constexpr int QT = 64;        // queries per CTA
constexpr int KT = 64;        // keys per tile
constexpr int LDS = 64 + 8;   // smem row stride in halves (144 B) to spread banks
constexpr float LOG2E = 1.4426950408889634f;

DEVI void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
DEVI void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
DEVI void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
DEVI uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Loads a 64-row tile of one head (Q or K columns) at segment positions [p0, p0+64), applies rotary if given
// (pairs i, i + HD/2), and stores fp16 into smem.  Rows past `limit` are zero.
template <int HD>
DEVI void load_tile_rope(__half* dst, const float* base, int ld, int p0, int limit, const float* cosv,
                         const float* sinv) {
    constexpr int HALF = HD / 2, J = HALF / 4;
    for (int it = threadIdx.x; it < 64 * J; it += blockDim.x) {
        const int r = it / J, j = it % J;
        const int pos = p0 + r;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
        if (pos < limit) {
            const float* src = base + static_cast<size_t>(pos) * ld;
            a = *reinterpret_cast<const float4*>(src + 4 * j);
            b = *reinterpret_cast<const float4*>(src + HALF + 4 * j);
            if (cosv) {
                const float4 c = *reinterpret_cast<const float4*>(cosv + static_cast<size_t>(pos) * HALF + 4 * j);
                const float4 s = *reinterpret_cast<const float4*>(sinv + static_cast<size_t>(pos) * HALF + 4 * j);
                float4 ra, rb;
                ra.x = __fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, s.x)); rb.x = __fadd_rn(__fmul_rn(b.x, c.x), __fmul_rn(a.x, s.x));
                ra.y = __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, s.y)); rb.y = __fadd_rn(__fmul_rn(b.y, c.y), __fmul_rn(a.y, s.y));
                ra.z = __fsub_rn(__fmul_rn(a.z, c.z), __fmul_rn(b.z, s.z)); rb.z = __fadd_rn(__fmul_rn(b.z, c.z), __fmul_rn(a.z, s.z));
                ra.w = __fsub_rn(__fmul_rn(a.w, c.w), __fmul_rn(b.w, s.w)); rb.w = __fadd_rn(__fmul_rn(b.w, c.w), __fmul_rn(a.w, s.w));
                a = ra; b = rb;
            }
        }
        uint2* da = reinterpret_cast<uint2*>(dst + r * LDS + 4 * j);
        uint2* db = reinterpret_cast<uint2*>(dst + r * LDS + HALF + 4 * j);
        *da = make_uint2(pack_half2(a.x, a.y), pack_half2(a.z, a.w));
        *db = make_uint2(pack_half2(b.x, b.y), pack_half2(b.z, b.w));
    }
}

template <int HD>
DEVI void load_tile_plain(__half* dst, const float* base, int ld, int p0, int limit) {
    constexpr int J = HD / 4;
    for (int it = threadIdx.x; it < 64 * J; it += blockDim.x) {
        const int r = it / J, j = it % J;
        const int pos = p0 + r;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        if (pos < limit) a = *reinterpret_cast<const float4*>(base + static_cast<size_t>(pos) * ld + 4 * j);
        *reinterpret_cast<uint2*>(dst + r * LDS + 4 * j) = make_uint2(pack_half2(a.x, a.y), pack_half2(a.z, a.w));
    }
}

template <int HD>
__global__ void __launch_bounds__(128) attention_kernel(Args a) {
    constexpr int KS = HD / 16;   // k-steps over the head dim
    constexpr int NT = HD / 8;    // 8-wide output tiles
    __shared__ __align__(16) __half Qs[QT * LDS];
    __shared__ __align__(16) __half Ks[KT * LDS];
    __shared__ __align__(16) __half Vs[KT * LDS];

    const int tile = blockIdx.x;
    if (tile >= *a.n_qtiles) return;
    const int head = blockIdx.y;
    const int item = a.qtile_item[tile];
    const int q0 = a.qtile_q0[tile];
    const int seg0 = a.seg_start[item];
    const int L = a.seg_len[item];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const bool global = a.window < 0;
    const int W = a.window;

    const float* qbase = a.qkv + static_cast<size_t>(seg0) * a.ld + head * HD;
    const float* kbase = qbase + a.hidden;
    const float* vbase = qbase + 2 * a.hidden;

    if (a.cosv) load_tile_rope<HD>(Qs, qbase, a.ld, q0, L, a.cosv, a.sinv);
    else load_tile_plain<HD>(Qs, qbase, a.ld, q0, L);

    const int kb = global ? 0 : max(0, q0 - W);
    const int ke = global ? L : min(L, q0 + QT + W);

    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.0f, 0.0f};
    const int qpos[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};

    uint32_t qa[KS][4];   // Q fragments for the warp's 16 rows, KS k-steps over the head dim
    __syncthreads();
    {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int c = ks * 16 + 8 * (lane >> 4);
            ldsm_x4(smem_u32(Qs + r * LDS + c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
        }
    }

    for (int k0 = kb; k0 < ke; k0 += KT) {
        __syncthreads();   // previous tile fully consumed
        if (a.cosv) load_tile_rope<HD>(Ks, kbase, a.ld, k0, ke, a.cosv, a.sinv);
        else load_tile_plain<HD>(Ks, kbase, a.ld, k0, ke);
        load_tile_plain<HD>(Vs, vbase, a.ld, k0, ke);
        __syncthreads();

        // S = Q Kᵀ for the warp's 16 rows × 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {   // pairs of 8-key n-tiles
                const int key = jp * 16 + (lane & 7) + 8 * (lane >> 4);
                const int dim = ks * 16 + 8 * ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(smem_u32(Ks + key * LDS + dim), b0, b1, b2, b3);
                mma16816(s[2 * jp], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
                mma16816(s[2 * jp + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
            }
        }
        // scale 1/√HD (AttentionKernels.Scores multiplies each dot by it), mask, online softmax
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int kp = k0 + 8 * j + 2 * t4 + (e & 1);
                const int qp = qpos[e >> 1];
                const bool ok = kp < ke && (global || (kp >= qp - W && kp <= qp + W));
                const float v = ok ? __fmul_rn(s[j][e], a.scale) : -INFINITY;
                s[j][e] = v;
                mx[e >> 1] = fmaxf(mx[e >> 1], v);
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        }
        float alpha[2], mnew[2], msc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mnew[h] = fmaxf(m_run[h], mx[h]);
            alpha[h] = (m_run[h] == -INFINITY) ? 0.0f : exp2f((m_run[h] - mnew[h]) * LOG2E);
            msc[h] = mnew[h] * LOG2E;
            m_run[h] = mnew[h];
        }
        float rs[2] = {0.0f, 0.0f};
        uint32_t pa[8][2];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int h = e >> 1;
                p[e] = (s[j][e] == -INFINITY) ? 0.0f : exp2f(fmaf(s[j][e], LOG2E, -msc[h]));
                rs[h] += p[e];
            }
            pa[j][0] = pack_half2(p[0], p[1]);
            pa[j][1] = pack_half2(p[2], p[3]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
            l_run[h] = l_run[h] * alpha[h] + rs[h];
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            o[j][0] *= alpha[0]; o[j][1] *= alpha[0];
            o[j][2] *= alpha[1]; o[j][3] *= alpha[1];
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {      // 16-key steps
#pragma unroll
            for (int dp = 0; dp < NT / 2; ++dp) {  // pairs of 8-dim n-tiles
                const int key = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int dim = dp * 16 + 8 * (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(smem_u32(Vs + key * LDS + dim), b0, b1, b2, b3);
                mma16816(o[2 * dp], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b0, b1);
                mma16816(o[2 * dp + 1], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b2, b3);
            }
        }
    }

    // Normalise, quantize to Q8_0 (two 32-dim blocks per head), store codes and scales — or, without a code buffer,
    // store the context split into hi/lo bf16 parts for a split product.
    if (a.q == nullptr) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int qp = qpos[h];
            if (qp >= L) continue;
            const float inv = l_run[h] > 0.0f ? 1.0f / l_run[h] : 0.0f;
            const size_t row = static_cast<size_t>(seg0 + qp) * a.hidden + head * HD;
#pragma unroll
            for (int j = 0; j < HD / 8; ++j) {
                const float v0 = o[j][2 * h] * inv, v1 = o[j][2 * h + 1] * inv;
                const __nv_bfloat16 h0 = __float2bfloat16_rn(v0), h1 = __float2bfloat16_rn(v1);
                const size_t c = row + 8 * j + 2 * t4;
                *reinterpret_cast<__nv_bfloat162*>(a.hi + c) = __halves2bfloat162(h0, h1);
                *reinterpret_cast<__nv_bfloat162*>(a.lo + c) =
                    __floats2bfloat162_rn(__fsub_rn(v0, __bfloat162float(h0)), __fsub_rn(v1, __bfloat162float(h1)));
            }
        }
        return;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int qp = qpos[h];
        const float inv = l_run[h] > 0.0f ? 1.0f / l_run[h] : 0.0f;
#pragma unroll
        for (int blk = 0; blk < HD / 32; ++blk) {
            float v[8];
            float m = 0.0f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                v[2 * jj] = o[blk * 4 + jj][2 * h] * inv;
                v[2 * jj + 1] = o[blk * 4 + jj][2 * h + 1] * inv;
                m = fmaxf(m, fmaxf(fabsf(v[2 * jj]), fabsf(v[2 * jj + 1])));
            }
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            const float id = m != 0.0f ? __fdiv_rn(127.0f, m) : 0.0f;
            if (qp < L) {
                const size_t tok = static_cast<size_t>(seg0 + qp);
                __half* qrow = a.q + tok * a.hidden + head * HD + blk * 32;
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int c0 = __float2int_rn(__fmul_rn(v[2 * jj], id));
                    const int c1 = __float2int_rn(__fmul_rn(v[2 * jj + 1], id));
                    *reinterpret_cast<__half2*>(qrow + 8 * jj + 2 * t4) = __halves2half2(__int2half_rn(c0), __int2half_rn(c1));
                }
                if (t4 == 0) a.d[static_cast<size_t>(head * (HD / 32) + blk) * a.ldd + tok] = round_fp16(__fdiv_rn(m, 127.0f));
            }
        }
    }
}

// One thread per 4 rotation pairs of one (token, head, q|k|v): the rotary of load_tile_rope, fp16 out.
__global__ void prep16_kernel(const float* __restrict__ src, int ld, int T, int hidden, int heads,
                              const int32_t* __restrict__ tok_item, const int32_t* __restrict__ seg_start,
                              const float* __restrict__ cosv, const float* __restrict__ sinv, __half* __restrict__ out,
                              int ldo) {
    constexpr int HD = 64, HALF = HD / 2, J = HALF / 4;
    const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<size_t>(T) * heads * 3 * J) return;
    const int j = static_cast<int>(idx % J);
    size_t rest = idx / J;
    const int part = static_cast<int>(rest % 3);
    rest /= 3;
    const int h = static_cast<int>(rest % heads);
    const int t = static_cast<int>(rest / heads);
    const int col = part * hidden + h * HD + 4 * j;
    float4 a = *reinterpret_cast<const float4*>(src + static_cast<size_t>(t) * ld + col);
    float4 b = *reinterpret_cast<const float4*>(src + static_cast<size_t>(t) * ld + col + HALF);
    if (part < 2 && cosv) {
        const int pos = t - seg_start[tok_item[t]];
        const float4 c = *reinterpret_cast<const float4*>(cosv + static_cast<size_t>(pos) * HALF + 4 * j);
        const float4 sn = *reinterpret_cast<const float4*>(sinv + static_cast<size_t>(pos) * HALF + 4 * j);
        float4 ra, rb;
        ra.x = __fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, sn.x)); rb.x = __fadd_rn(__fmul_rn(b.x, c.x), __fmul_rn(a.x, sn.x));
        ra.y = __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, sn.y)); rb.y = __fadd_rn(__fmul_rn(b.y, c.y), __fmul_rn(a.y, sn.y));
        ra.z = __fsub_rn(__fmul_rn(a.z, c.z), __fmul_rn(b.z, sn.z)); rb.z = __fadd_rn(__fmul_rn(b.z, c.z), __fmul_rn(a.z, sn.z));
        ra.w = __fsub_rn(__fmul_rn(a.w, c.w), __fmul_rn(b.w, sn.w)); rb.w = __fadd_rn(__fmul_rn(b.w, c.w), __fmul_rn(a.w, sn.w));
        a = ra; b = rb;
    }
    __half* d = out + static_cast<size_t>(t) * ldo + col;
    *reinterpret_cast<uint2*>(d) = make_uint2(pack_half2(a.x, a.y), pack_half2(a.z, a.w));
    *reinterpret_cast<uint2*>(d + HALF) = make_uint2(pack_half2(b.x, b.y), pack_half2(b.z, b.w));
}

}  // namespace attn

int attn_prep16(const float* qkv, int ld, int T, int hidden, int heads, const int32_t* tok_item, const int32_t* seg_start,
                const float* cosv, const float* sinv, __half* out, int ldo, cudaStream_t stream) {
    if (T <= 0) return OK;
    if (hidden != 64 * heads || (ld & 3) || (ldo & 7)) { set_error("fp16 attention prep: head_dim 64, aligned rows"); return ERR_ARGUMENT; }
    const size_t n = static_cast<size_t>(T) * heads * 3 * 8;
    attn::prep16_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(qkv, ld, T, hidden, heads, tok_item,
                                                                                   seg_start, cosv, sinv, out, ldo);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int attention(const attn::Args& a, int max_qtiles, cudaStream_t stream) {
    if (max_qtiles <= 0) return OK;
    dim3 grid(max_qtiles, a.heads);
    const int hd = a.heads > 0 ? a.hidden / a.heads : 0;
    if (hd * a.heads != a.hidden) { set_error("hidden is not a multiple of the head count"); return ERR_ARGUMENT; }
    if (hd == 64) attn::attention_kernel<64><<<grid, 128, 0, stream>>>(a);
    else if (hd == 32) attn::attention_kernel<32><<<grid, 128, 0, stream>>>(a);
    else { set_error("attention kernels support head_dim 32 and 64"); return ERR_NOT_SUPPORTED; }
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace laya
