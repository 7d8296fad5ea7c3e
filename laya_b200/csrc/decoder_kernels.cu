// decoder_kernels.cu — the Mica decoder's (Qwen3.5 hybrid) kernels other than the Q8_0 products (q8_gemm.cu).
//
// Replaces DecoderKernels (Base/Numerics/DecoderKernels.cs) and the per-token loops of Qwen35Model
// (Mica/Models/Qwen35Model.cs):
//   rms_q8          RMSNorm (scale = 1 + weight) fused with the Q8_0 activation quantizer of the next product;
//                   SumOfSquares by 8 lane FMA chains and the reference's fixed combine, so the codes are the
//                   CPU restatement's bits (DecoderKernels.cs:15-46, PackedMatrixQ8_0.cs:35-71)
//   embed           TokenTable.Row of a Q8_0 table: code · block scale (Qwen35Model.cs:1070-1082)
//   conv_silu       the DeltaNet's causal depthwise conv (taps summed in order, multiply then add) + SiLU
//   deltanet_heads  L2 norm of q (· 1/sqrt(dk)) and k per key head, β = sigmoid(b), g = exp(−e^A·softplus(a+dt))
//   delta_rule      the gated delta rule, one CTA per (sequence, value head), thread j owning state column j;
//                   the fused single sweep of DecoderKernels.GatedDeltaRule128 (bit-identical to the two-sweep
//                   recurrence of Qwen35Model.Recurrence, Qwen35Model.cs:924-972)
//   gated_norm      RmsNormGated: weight · rmsnorm(o) · silu(z) per value head (DecoderKernels.cs:52-64)
//   attn_prep       per-head RMSNorm of q and k + rotate-half RoPE on the first rotary dims; fp16 q, k, v
//   attention       causal GQA softmax attention, fp16 mma.sync tiles with fp32 softmax, · sigmoid(gate)
//   q8_logits       TokenTable.QuantizedLogits: per block an exact integer dot, fma((float)Σ, d_w·d_x, acc)
#include <algorithm>

#include "common.cuh"
#include "decoder.h"
#include "internal.h"

namespace laya {
namespace dec {

using q8::code_t;

DEVI float octet_hsum(float a) {   // (a0+a4, a1+a5, a2+a6, a3+a7) then pairwise, as the CPU restatement
    float t = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
    float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
    return __fadd_rn(u, __shfl_xor_sync(0xffffffffu, u, 2));
}
DEVI float octet_max(float a) {
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    return fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
}

// Q8_0 of 32 values held 4 per octet lane (lane l: elements l, l+8, l+16, l+24 of the block).
DEVI void quantize_octet_block(const float (&v)[4], code_t* qrow, float* dslot, int l, bool active) {
    float m = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) m = fmaxf(m, fabsf(v[t]));
    const float amax = octet_max(m);
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    if (active) {
#pragma unroll
        for (int t = 0; t < 4; ++t) qrow[l + 8 * t] = __int2half_rn(__float2int_rn(__fmul_rn(v[t], id)));
        if (l == 0) *dslot = round_fp16(__fdiv_rn(amax, 127.0f));
    }
}

// ------------------------------------------------------------------------------------------------ RMSNorm → Q8_0
__global__ void __launch_bounds__(256) rms_q8_kernel(RmsArgs a) {
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = gt >> 3, l = gt & 7;
    const bool active = row < a.rows;
    const int r = active ? row : a.rows - 1;
    const int src_row = a.row_map ? a.row_map[r] : r;
    const float* x = a.x + static_cast<size_t>(src_row) * a.n;
    float ss = 0.0f;
    for (int i = l; i < a.n; i += 8) ss = __fmaf_rn(x[i], x[i], ss);
    ss = octet_hsum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(a.n)), a.eps)));
    for (int b = 0; b < a.n / 32; ++b) {
        float v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int c = b * 32 + l + 8 * t;
            v[t] = __fmul_rn(__fmul_rn(x[c], inv), a.scale[c]);
            if (a.out32 && active) a.out32[static_cast<size_t>(r) * a.n + c] = v[t];
        }
        if (a.q) quantize_octet_block(v, a.q + static_cast<size_t>(r) * a.n + b * 32, a.d + static_cast<size_t>(b) * a.ldd + r, l, active);
    }
}

// ------------------------------------------------------------------------------------------------ embeddings
__global__ void embed_kernel(const int32_t* __restrict__ ids, int T, int n, int vocab, const code_t* __restrict__ q,
                             const float* __restrict__ d, int ldd, float* __restrict__ x, int* err) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(T) * n) return;
    const int t = static_cast<int>(i / n), c = static_cast<int>(i % n);
    int id = ids[t];
    if (id < 0 || id >= vocab) {
        if (c == 0) atomicExch(err, LAYA_DEV_ERR_BOUNDS);
        id = 0;
    }
    x[i] = __fmul_rn(__half2float(q[static_cast<size_t>(id) * n + c]), d[static_cast<size_t>(c / 32) * ldd + id]);
}

// ------------------------------------------------------------------------------------------------ DeltaNet
// conv[t, c] = silu(Σ_j w[j, c] · in[t − (K−1) + j, c]) over t's sequence history: its rows, preceded by the K−1 rows
// of its state's conv tail (zero without a state).
// Thread = one channel over a run of CONV_RUN consecutive tokens: each input is read once (coalesced across
// channels) and the last K−1 inputs ride along in registers; taps before the token's sequence start read the tail.
DEVI float conv_history(const ConvArgs& a, int seq, int before, int c) {   // before ∈ [−(K−1), −1]
    const float* tail = a.tails ? a.tails[seq] : nullptr;
    return tail ? tail[static_cast<size_t>(a.K - 1 + before) * a.cd + c] : 0.0f;
}
constexpr int CONV_RUN = 32;
template <int K>
__global__ void __launch_bounds__(256) conv_silu_kernel(ConvArgs a) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int t0 = blockIdx.y * CONV_RUN;
    if (c >= a.cd) return;
    const int t1 = min(a.T, t0 + CONV_RUN);
    float w[K], h[K];
#pragma unroll
    for (int j = 0; j < K; ++j) w[j] = a.w[static_cast<size_t>(j) * a.cd + c];
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {   // h[j] = in[t0 − (K−1) + j]; the mask below drops rows before a sequence start
        const int src = t0 - (K - 1) + j;
        h[j] = src >= 0 ? a.in[static_cast<size_t>(src) * a.ld_in + c] : 0.0f;
    }
    for (int t = t0; t < t1; ++t) {
        h[K - 1] = a.in[static_cast<size_t>(t) * a.ld_in + c];
        const int seq = a.tok_seq[t];
        const int s0 = a.seq_start[seq];
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int src = t - (K - 1) + j;
            sum = __fadd_rn(sum, __fmul_rn(w[j], src >= s0 ? h[j] : conv_history(a, seq, src - s0, c)));
        }
        a.out[static_cast<size_t>(t) * a.cd + c] = ref_silu(sum);
#pragma unroll
        for (int j = 0; j < K - 1; ++j) h[j] = h[j + 1];
    }
}
// Any kernel size: one thread per (token, channel).
__global__ void conv_silu_any_kernel(ConvArgs a) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(a.T) * a.cd) return;
    const int t = static_cast<int>(i / a.cd), c = static_cast<int>(i % a.cd);
    const int seq = a.tok_seq[t];
    const int s0 = a.seq_start[seq];
    float sum = 0.0f;
    for (int j = 0; j < a.K; ++j) {
        const int src = t - (a.K - 1) + j;
        const float h = src >= s0 ? a.in[static_cast<size_t>(src) * a.ld_in + c] : conv_history(a, seq, src - s0, c);
        sum = __fadd_rn(sum, __fmul_rn(a.w[static_cast<size_t>(j) * a.cd + c], h));
    }
    a.out[i] = ref_silu(sum);
}

// Thread = (sequence, channel): the snapshots' tails (history rows [cp − (K−1), cp) of the read), then the state's own
// tail (rows [L − (K−1), L)), history row r < 0 being row K−1+r of the old tail.  The own tail is rewritten in place in
// ascending order: row j reads old row L + j > j, not yet overwritten (Qwen35Model.cs:814-830).
__global__ void __launch_bounds__(256) conv_state_kernel(ConvStateArgs a) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, seq = blockIdx.y;
    if (c >= a.cd) return;
    float* tail = a.tails[seq];
    if (!tail) return;
    const int s0 = a.seq_start[seq], L = a.seq_len[seq], keep = a.K - 1;
    auto hist = [&](int r) {
        return r >= 0 ? a.in[static_cast<size_t>(s0 + r) * a.ld_in + c] : tail[static_cast<size_t>(keep + r) * a.cd + c];
    };
    if (a.snap_begin) {
        for (int k = a.snap_begin[seq]; k < a.snap_begin[seq + 1]; ++k) {
            float* dst = a.snap_tails[k];
            const int cp = a.snap_at[k];
            for (int j = 0; j < keep; ++j) dst[static_cast<size_t>(j) * a.cd + c] = hist(cp - keep + j);
        }
    }
    for (int j = 0; j < keep; ++j) tail[static_cast<size_t>(j) * a.cd + c] = hist(L - keep + j);
}

// One octet per (token, key head, q|k): L2Normalize (DecoderKernels.cs:67-85); plus β and g per value head.
__global__ void __launch_bounds__(256) deltanet_heads_kernel(HeadsArgs a) {
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    const int item = gt >> 3, l = gt & 7;
    const int per_tok = 2 * a.kh;
    const bool active = item < a.T * per_tok;
    const int it = active ? item : a.T * per_tok - 1;
    const int t = it / per_tok, w = it % per_tok;
    const int which = w / a.kh, h = w % a.kh;   // 0: q, 1: k
    float* v = a.conv + static_cast<size_t>(t) * a.cd + which * a.key_dim + h * a.dk;
    float ss = 0.0f;
    for (int i = l; i < a.dk; i += 8) ss = __fmaf_rn(v[i], v[i], ss);
    ss = octet_hsum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, 1e-6f)));
    const float extra = which == 0 ? a.qscale : 1.0f;
    __syncwarp();
    if (active)
        for (int i = l; i < a.dk; i += 8) {
            const float x = __fmul_rn(v[i], inv);
            v[i] = extra != 1.0f ? __fmul_rn(x, extra) : x;
        }
    // gates: the first T·vh threads of the grid, one per (token, value head)
    if (gt < a.T * a.vh) {
        const int tt = gt / a.vh, hh = gt % a.vh;
        const float b = a.proj[static_cast<size_t>(tt) * a.ld_proj + a.b_col + hh];
        const float av = a.proj[static_cast<size_t>(tt) * a.ld_proj + a.a_col + hh];
        a.beta[gt] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b)));
        const float xs = __fadd_rn(av, a.dt_bias[hh]);
        const float sp = xs > 20.0f ? xs : static_cast<float>(log1p(exp(static_cast<double>(xs))));
        const float g = expf(__fmul_rn(a.neg_a[hh], sp));
        a.decay[gt] = g < 1.17549435e-38f ? 0.0f : g;   // subnormal decays flush to 0 (Qwen35Model.cs:866-873)
    }
}

// The gated delta rule of one (sequence, value head).  Thread j < dv owns state column S[:, j] (DK registers).
// The CTA stages q, k, v, β and the decay of CH tokens (plus the next token's k and decay) in shared memory with
// cp.async, double-buffered: the next chunk loads while this one runs, so a token's step waits on no global load.
//   token 0:    S ← S·g_0;  m = Sᵀk_0            (S: the sequence's state, or zero)
//   token t:    δ = (v_t − m)·β_t;  for i: x = S_i + δ·k_t,i (fma);  o += x·q_t,i (fma);  S_i = x·g_{t+1};
//               m' += S_i·k_{t+1},i (fma)          (the last token skips the decay and the next read)
// A checkpoint after token t splits that fused step into the same operations in the same order: the update, the copy
// of S to the snapshot, then the next token's decay and read.  The final S goes back to the state.
DEVI void cp16(float* dst, const float* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
DEVI void cp4(float* dst, const float* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
DEVI void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
DEVI void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int RULE_CH = 16, RULE_DV = 128;
template <int DK>
struct RuleSmem {   // one buffer, in floats
    static constexpr int Q = 0, K = RULE_CH * DK, V = K + (RULE_CH + 1) * DK, B = V + RULE_CH * RULE_DV,
                         G = B + RULE_CH, SIZE = (G + RULE_CH + 1 + 3) / 4 * 4;
};

template <int DK>
__global__ void __launch_bounds__(128) delta_rule_kernel(DeltaArgs a) {
    constexpr int CH = RULE_CH;
    using SM = RuleSmem<DK>;
    extern __shared__ __align__(16) float rsm[];
    const int seq = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
    const int kh = h / a.ratio;
    const int s0 = a.seq_start[seq], L = a.seq_len[seq];
    const bool act = j < a.dv;
    const float* base = a.conv + static_cast<size_t>(s0) * a.cd;
    const int qoff = kh * DK, koff = a.key_dim + kh * DK, voff = 2 * a.key_dim + h * a.dv;
    const int nch = (L + CH - 1) / CH;
    const int dv4 = a.dv / 4;

    auto issue = [&](int c, float* buf) {
        const int t0 = c * CH, n = min(CH, L - t0);
        for (int e = threadIdx.x; e < (CH + 1) * (DK / 4); e += blockDim.x) {
            const int r = e / (DK / 4), c4 = e % (DK / 4);
            const bool kin = t0 + r < L, qin = r < n;
            const float* row = base + static_cast<size_t>(kin ? t0 + r : 0) * a.cd;
            cp16(buf + SM::K + r * DK + 4 * c4, row + koff + 4 * c4, kin);
            if (r < CH) cp16(buf + SM::Q + r * DK + 4 * c4, row + qoff + 4 * c4, qin);
        }
        for (int e = threadIdx.x; e < CH * dv4; e += blockDim.x) {
            const int r = e / dv4, c4 = e % dv4;
            const bool in = r < n;
            cp16(buf + SM::V + r * RULE_DV + 4 * c4, base + static_cast<size_t>(in ? t0 + r : 0) * a.cd + voff + 4 * c4, in);
        }
        for (int r = threadIdx.x; r <= CH; r += blockDim.x) {
            const bool gin = t0 + r < L, bin = r < n;
            const size_t row = static_cast<size_t>(s0 + (gin ? t0 + r : 0)) * a.vh + h;
            cp4(buf + SM::G + r, a.decay + row, gin);
            if (r < CH) cp4(buf + SM::B + r, a.beta + row, bin);
        }
        cp_commit();
    };

    const size_t head_off = static_cast<size_t>(h) * DK * a.dv;
    float* rec = a.rec ? a.rec[seq] : nullptr;
    float s[DK];
#pragma unroll
    for (int i = 0; i < DK; ++i) s[i] = (rec && act) ? rec[head_off + static_cast<size_t>(i) * a.dv + j] : 0.0f;
    int sk = a.snap_begin ? a.snap_begin[seq] : 0;
    const int se = a.snap_begin ? a.snap_begin[seq + 1] : 0;
    int next_cp = sk < se ? a.snap_at[sk] : -1;   // token count of the next checkpoint
    int stop = next_cp > 0 ? next_cp : L;          // the fused step runs while t + 1 < stop
    float m = 0.0f;
    issue(0, rsm);
    for (int c = 0; c < nch; ++c) {
        const float* cur = rsm + (c & 1) * SM::SIZE;
        if (c + 1 < nch) {
            issue(c + 1, rsm + ((c + 1) & 1) * SM::SIZE);
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const float* qs = cur + SM::Q;
        const float* ks = cur + SM::K;
        const int t0 = c * CH, n = min(CH, L - t0);
        if (c == 0) {   // token 0's decay and read
            const float g = cur[SM::G];
#pragma unroll
            for (int i = 0; i < DK; ++i) {
                s[i] = __fmul_rn(s[i], g);
                m = __fmaf_rn(s[i], ks[i], m);
            }
        }
        for (int r = 0; r < n; ++r) {
            const int t = t0 + r;
            const float v = act ? cur[SM::V + r * RULE_DV + j] : 0.0f;
            const float d = __fmul_rn(__fsub_rn(v, m), cur[SM::B + r]);
            const float* kr = ks + r * DK;
            const float* qr = qs + r * DK;
            float o = 0.0f;
            // Every warp reads the same q and k values (shared-memory broadcasts, one 4-byte value per wavefront):
            // with 4 warps that is 3·DK·4 wavefronts per token, which bounds this exact sequential form.
            if (t + 1 < stop) {
                const float g = cur[SM::G + r + 1];
                const float* kn = kr + DK;
                float mn = 0.0f;
#pragma unroll
                for (int i = 0; i < DK; ++i) {
                    float x = __fmaf_rn(d, kr[i], s[i]);
                    o = __fmaf_rn(x, qr[i], o);
                    x = __fmul_rn(x, g);
                    s[i] = x;
                    mn = __fmaf_rn(x, kn[i], mn);
                }
                m = mn;
            } else {
#pragma unroll
                for (int i = 0; i < DK; ++i) {
                    const float x = __fmaf_rn(d, kr[i], s[i]);
                    o = __fmaf_rn(x, qr[i], o);
                    s[i] = x;
                }
                if (t + 1 == next_cp) {   // the same for every thread of the CTA
                    float* dst = a.snap_rec[sk] + head_off;
                    if (act) {
#pragma unroll
                        for (int i = 0; i < DK; ++i) dst[static_cast<size_t>(i) * a.dv + j] = s[i];
                    }
                    ++sk;
                    next_cp = sk < se ? a.snap_at[sk] : -1;
                    stop = next_cp > 0 ? next_cp : L;
                    if (t + 1 < L) {   // the next token's decay and read (staged: k and g of row r + 1 ≤ CH)
                        const float g = cur[SM::G + r + 1];
                        const float* kn = kr + DK;
                        float mn = 0.0f;
#pragma unroll
                        for (int i = 0; i < DK; ++i) {
                            s[i] = __fmul_rn(s[i], g);
                            mn = __fmaf_rn(s[i], kn[i], mn);
                        }
                        m = mn;
                    }
                }
            }
            if (act) a.out[static_cast<size_t>(s0 + t) * a.ld_out + h * a.dv + j] = o;
        }
        __syncthreads();
    }
    if (rec && act) {
#pragma unroll
        for (int i = 0; i < DK; ++i) rec[head_off + static_cast<size_t>(i) * a.dv + j] = s[i];
    }
}

// RmsNormGated per (token, value head) octet; output fp32 (quantized afterwards, blocks span heads).
__global__ void __launch_bounds__(256) gated_norm_kernel(GatedArgs a) {
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    const int item = gt >> 3, l = gt & 7;
    const bool active = item < a.T * a.vh;
    const int it = active ? item : a.T * a.vh - 1;
    const int t = it / a.vh, h = it % a.vh;
    const float* o = a.core + static_cast<size_t>(t) * a.ld_core + h * a.dv;
    const float* z = a.z + static_cast<size_t>(t) * a.ld_z + h * a.dv;
    float ss = 0.0f;
    for (int i = l; i < a.dv; i += 8) ss = __fmaf_rn(o[i], o[i], ss);
    ss = octet_hsum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(a.dv)), a.eps)));
    if (!active) return;
    float* y = a.out + static_cast<size_t>(t) * a.ld_out + h * a.dv;
    for (int i = l; i < a.dv; i += 8)
        y[i] = __fmul_rn(__fmul_rn(a.weight[i], __fmul_rn(o[i], inv)), ref_silu(z[i]));
}

// ------------------------------------------------------------------------------------------------ full attention
// One warp per 4 (token, head) items, an octet each: RMSNorm over head_dim (1 + w), then rotate-half on the first
// 2·half dims from a warp-private shared copy; q, k to fp16, v copied.
__global__ void __launch_bounds__(256) attn_prep_kernel(PrepArgs a) {
    extern __shared__ float sh[];   // [8 warps][4 octets][hd]
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    const int item = gt >> 3, l = gt & 7, oct = (threadIdx.x >> 3) & 3, warp = threadIdx.x >> 5;
    const int per_tok = a.heads + a.kv_heads;
    const bool active = item < a.T * per_tok;
    const int it = active ? item : a.T * per_tok - 1;
    const int t = it / per_tok, w = it % per_tok;
    const bool isq = w < a.heads;
    const int h = isq ? w : w - a.heads;
    const float* src = a.qkv + static_cast<size_t>(t) * a.ld_qkv + (isq ? h * 2 * a.hd : a.q_width + h * a.hd);
    const float* sc = isq ? a.qnorm : a.knorm;
    float ss = 0.0f;
    for (int i = l; i < a.hd; i += 8) ss = __fmaf_rn(src[i], src[i], ss);
    ss = octet_hsum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(a.hd)), a.eps)));
    float* buf = sh + (warp * 4 + oct) * a.hd;
    for (int i = l; i < a.hd; i += 8) buf[i] = __fmul_rn(__fmul_rn(src[i], inv), sc[i]);
    __syncwarp();
    const int seq = a.tok_seq[t];
    const int pos = a.pos0[seq] + t - a.seq_start[seq];
    const size_t kv_row = static_cast<size_t>(pos) * a.kv_heads * a.hd + h * a.hd;
    __half* dst = isq ? a.q16 + static_cast<size_t>(t) * a.heads * a.hd + h * a.hd : a.kc[seq] + kv_row;
    if (active) {
        for (int i = l; i < a.hd; i += 8) {
            float y = buf[i];
            if (i < 2 * a.half) {
                const int p = i < a.half ? i : i - a.half;
                const float c = a.cosv[static_cast<size_t>(pos) * a.half + p], s = a.sinv[static_cast<size_t>(pos) * a.half + p];
                y = i < a.half ? __fsub_rn(__fmul_rn(buf[i], c), __fmul_rn(buf[i + a.half], s))
                               : __fadd_rn(__fmul_rn(buf[i], c), __fmul_rn(buf[i - a.half], s));
            }
            dst[i] = __float2half_rn(y);
        }
        if (!isq) {
            const float* vs = a.qkv + static_cast<size_t>(t) * a.ld_qkv + a.q_width + a.kv_heads * a.hd + h * a.hd;
            __half* vd = a.vc[seq] + kv_row;
            for (int i = l; i < a.hd; i += 8) vd[i] = __float2half_rn(vs[i]);
        }
    }
}

// Causal GQA attention, 64 queries × 64 keys per step, 4 warps × 16 rows, fp16 mma.sync → fp32.
constexpr int T64 = 64;
DEVI void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
DEVI void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
DEVI void mma_f16_sync(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
DEVI uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int HD>
__global__ void __launch_bounds__(128) attention_kernel(AttnArgs a) {
    constexpr int LDS = HD + 8, KS = HD / 16, NT = HD / 8;
    extern __shared__ __align__(16) __half asm_[];
    __half* Qs = asm_;
    __half* Ks = Qs + T64 * LDS;
    __half* Vs = Ks + T64 * LDS;
    const int tile = blockIdx.x;
    const int head = blockIdx.y, kvh = head / (a.heads / a.kv_heads);
    const int seq = a.tile_seq[tile], q0 = a.tile_p0[tile];
    const int s0 = a.seq_start[seq], L = a.seq_len[seq], P = a.pos0[seq];   // queries: positions P + [0, L)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const int ldq = a.heads * HD, ldkv = a.kv_heads * HD;
    // rows p0 .. p0+63 of src (row stride ld), those < limit; the rest zero
    auto load = [&](__half* dst, const __half* src, int ld, int p0, int limit) {
        constexpr int CH = HD / 8;
        for (int e = threadIdx.x; e < T64 * CH; e += blockDim.x) {
            const int r = e / CH, c = e % CH;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (p0 + r < limit) v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(p0 + r) * ld + c * 8);
            *reinterpret_cast<uint4*>(dst + r * LDS + c * 8) = v;
        }
    };
    load(Qs, a.q16 + static_cast<size_t>(s0) * ldq + head * HD, ldq, q0, L);
    __syncthreads();
    uint32_t fq[KS][4];
    {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks)
            ldsm_x4(smem_u32(Qs + r * LDS + ks * 16 + 8 * (lane >> 4)), fq[ks][0], fq[ks][1], fq[ks][2], fq[ks][3]);
    }
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const int qp[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};   // rows of the read
    const int ke = P + min(L, q0 + T64);   // causal: key positions up to the tile's last query
    const __half* kbase = a.kc[seq] + kvh * HD;
    const __half* vbase = a.vc[seq] + kvh * HD;
    // Key tiles start at position 0 whatever P is, so a row's softmax runs over the same tiles in the same order as
    // when its sequence is read in one pass (tiles past the row are fully masked and change nothing).
    for (int k0 = 0; k0 < ke; k0 += T64) {
        __syncthreads();
        load(Ks, kbase, ldkv, k0, P + L);
        load(Vs, vbase, ldkv, k0, P + L);
        __syncthreads();
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                const int row = jp * 16 + (lane & 7) + 8 * (lane >> 4);
                const int col = ks * 16 + 8 * ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(smem_u32(Ks + row * LDS + col), b0, b1, b2, b3);
                mma_f16_sync(s[2 * jp], fq[ks][0], fq[ks][1], fq[ks][2], fq[ks][3], b0, b1);
                mma_f16_sync(s[2 * jp + 1], fq[ks][0], fq[ks][1], fq[ks][2], fq[ks][3], b2, b3);
            }
        }
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int kp = k0 + 8 * j + 2 * t4 + (e & 1);
                const int q = qp[e >> 1];
                const float v = (kp <= P + q && q < L) ? __fmul_rn(s[j][e], a.scale) : -INFINITY;
                s[j][e] = v;
                mx[e >> 1] = fmaxf(mx[e >> 1], v);
            }
        float alpha[2], msc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
            const float mn = fmaxf(m_run[h], mx[h]);
            alpha[h] = m_run[h] == -INFINITY ? 0.f : __expf(m_run[h] - mn);
            msc[h] = mn == -INFINITY ? 0.f : mn;
            m_run[h] = mn;
        }
        float rs[2] = {0.f, 0.f};
        uint32_t pa[8][2];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float pv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float pe = s[j][e] == -INFINITY ? 0.f : __expf(s[j][e] - msc[e >> 1]);
                rs[e >> 1] += pe;
                pv[e] = pe;
            }
            pa[j][0] = pack_h2(pv[0], pv[1]);
            pa[j][1] = pack_h2(pv[2], pv[3]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
            l_run[h] = l_run[h] * alpha[h] + rs[h];
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) { o[j][0] *= alpha[0]; o[j][1] *= alpha[0]; o[j][2] *= alpha[1]; o[j][3] *= alpha[1]; }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int dp = 0; dp < NT / 2; ++dp) {
                const int row = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int col = dp * 16 + 8 * (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(smem_u32(Vs + row * LDS + col), b0, b1, b2, b3);
                mma_f16_sync(o[2 * dp], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b0, b1);
                mma_f16_sync(o[2 * dp + 1], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], b2, b3);
            }
        }
    }
    // · sigmoid(gate) (DecoderKernels.MultiplySigmoid), fp32 out
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int q = qp[h];
        if (q >= L) continue;
        const float inv = l_run[h] > 0.f ? 1.0f / l_run[h] : 0.f;
        const size_t t = static_cast<size_t>(s0 + q);
        const float* gate = a.qkv + t * a.ld_qkv + head * 2 * HD + HD;
        float* orow = a.out + t * a.ld_out + head * HD;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int d = 8 * j + 2 * t4;
            orow[d] = __fmul_rn(o[j][2 * h] * inv, ref_sigmoid(gate[d]));
            orow[d + 1] = __fmul_rn(o[j][2 * h + 1] * inv, ref_sigmoid(gate[d + 1]));
        }
    }
}

// dst[r, :n] = src[map[r], :n] (the readout rows of the last layer)
__global__ void gather_rows_kernel(const float* __restrict__ src, int ld_src, const int32_t* __restrict__ map, int rows,
                                   int n, float* __restrict__ dst, int ld_dst) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(rows) * n) return;
    const int r = static_cast<int>(i / n), c = static_cast<int>(i % n);
    dst[static_cast<size_t>(r) * ld_dst + c] = src[static_cast<size_t>(map[r]) * ld_src + c];
}

// x += y elementwise (the residual add behind a recorded mixer or MLP output; the same single rounding as the
// product's residual epilogue).
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], y[i]);
}

// ------------------------------------------------------------------------------------------------ logits
// One warp per (sequence, label): lanes take the integer block dots, lane 0 folds them in block order.
__global__ void q8_logits_kernel(LogitArgs a) {
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (gw >= a.n_seq * a.n_labels) return;
    const int s = gw / a.n_labels, li = gw % a.n_labels;
    int id = a.labels[li];
    if (id < 0 || id >= a.vocab) {
        if (lane == 0) atomicExch(a.err, LAYA_DEV_ERR_BOUNDS);
        id = 0;
    }
    const int nb = a.n / 32;
    float acc = 0.0f;
    for (int b0 = 0; b0 < nb; b0 += 32) {
        const int b = b0 + lane;
        int sum = 0;
        if (b < nb) {
            const code_t* x = a.qx + static_cast<size_t>(s) * a.n + b * 32;
            const code_t* w = a.qw + static_cast<size_t>(id) * a.n + b * 32;
#pragma unroll 8
            for (int k = 0; k < 32; ++k) sum += __half2int_rn(x[k]) * __half2int_rn(w[k]);
        }
        const float scale = b < nb ? __fmul_rn(a.dw[static_cast<size_t>(b) * a.ldw + id], a.dx[static_cast<size_t>(b) * a.ldx + s]) : 0.0f;
        for (int k = 0; k < 32 && b0 + k < nb; ++k) {
            const int sk = __shfl_sync(0xffffffffu, sum, k);
            const float ck = __shfl_sync(0xffffffffu, scale, k);
            acc = __fmaf_rn(static_cast<float>(sk), ck, acc);
        }
    }
    if (lane == 0) a.logits[gw] = acc;
}

}  // namespace dec

// ------------------------------------------------------------------------------------------------ launchers
static unsigned nblk(size_t n, int t) { return static_cast<unsigned>((n + t - 1) / t); }
#define DEC_LAUNCHED()                 \
    do {                               \
        count_launch();                \
        LAYA_CUDA(cudaGetLastError()); \
        return OK;                     \
    } while (0)

int dec_rms_q8(const dec::RmsArgs& a, cudaStream_t s) {
    if (a.rows <= 0) return OK;
    if (a.n % 32) { set_error("RMSNorm width must be a multiple of 32"); return ERR_NOT_SUPPORTED; }
    dec::rms_q8_kernel<<<nblk(static_cast<size_t>(a.rows) * 8, 256), 256, 0, s>>>(a);
    DEC_LAUNCHED();
}
int dec_embed(const int32_t* ids, int T, int n, int vocab, const q8::code_t* q, const float* d, int ldd, float* x,
              int* err, cudaStream_t s) {
    if (T <= 0) return OK;
    dec::embed_kernel<<<nblk(static_cast<size_t>(T) * n, 256), 256, 0, s>>>(ids, T, n, vocab, q, d, ldd, x, err);
    DEC_LAUNCHED();
}
int dec_conv_silu(const dec::ConvArgs& a, cudaStream_t s) {
    if (a.T <= 0) return OK;
    const dim3 grid((a.cd + 255) / 256, (a.T + dec::CONV_RUN - 1) / dec::CONV_RUN);
    switch (a.K) {
        case 2: dec::conv_silu_kernel<2><<<grid, 256, 0, s>>>(a); break;
        case 3: dec::conv_silu_kernel<3><<<grid, 256, 0, s>>>(a); break;
        case 4: dec::conv_silu_kernel<4><<<grid, 256, 0, s>>>(a); break;
        default: dec::conv_silu_any_kernel<<<nblk(static_cast<size_t>(a.T) * a.cd, 256), 256, 0, s>>>(a); break;
    }
    DEC_LAUNCHED();
}
int dec_conv_state(const dec::ConvStateArgs& a, cudaStream_t s) {
    if (a.n_seq <= 0 || a.K < 2) return OK;
    dec::conv_state_kernel<<<dim3((a.cd + 255) / 256, a.n_seq), 256, 0, s>>>(a);
    DEC_LAUNCHED();
}
int dec_deltanet_heads(const dec::HeadsArgs& a, cudaStream_t s) {
    if (a.T <= 0) return OK;
    const size_t threads = std::max(static_cast<size_t>(a.T) * 2 * a.kh * 8, static_cast<size_t>(a.T) * a.vh);
    dec::deltanet_heads_kernel<<<nblk(threads, 256), 256, 0, s>>>(a);
    DEC_LAUNCHED();
}
int dec_delta_rule(const dec::DeltaArgs& a, int n_seq, cudaStream_t s) {
    if (n_seq <= 0) return OK;
    const int chunked = dec_delta_rule_chunked(a, n_seq, s);   // 64-token chunks on the tensor cores where it applies
    if (chunked != ERR_NOT_SUPPORTED) return chunked;
    if (a.dv > dec::RULE_DV || a.dv % 4) { set_error("delta rule: value head dim must be a multiple of 4, at most 128"); return ERR_NOT_SUPPORTED; }
    const dim3 grid(n_seq, a.vh);
    const int threads = (a.dv + 31) / 32 * 32;
    auto run = [&](auto kern, int floats) -> int {
        const int bytes = 2 * floats * static_cast<int>(sizeof(float));
        LAYA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        kern<<<grid, threads, bytes, s>>>(a);
        return OK;
    };
    int rc;
    switch (a.dk) {
        case 16: rc = run(dec::delta_rule_kernel<16>, dec::RuleSmem<16>::SIZE); break;
        case 32: rc = run(dec::delta_rule_kernel<32>, dec::RuleSmem<32>::SIZE); break;
        case 64: rc = run(dec::delta_rule_kernel<64>, dec::RuleSmem<64>::SIZE); break;
        case 128: rc = run(dec::delta_rule_kernel<128>, dec::RuleSmem<128>::SIZE); break;
        default: set_error("delta rule: key head dim must be 16, 32, 64 or 128"); return ERR_NOT_SUPPORTED;
    }
    if (rc != OK) return rc;
    DEC_LAUNCHED();
}
int dec_gated_norm(const dec::GatedArgs& a, cudaStream_t s) {
    if (a.T <= 0) return OK;
    dec::gated_norm_kernel<<<nblk(static_cast<size_t>(a.T) * a.vh * 8, 256), 256, 0, s>>>(a);
    DEC_LAUNCHED();
}
int dec_attn_prep(const dec::PrepArgs& a, cudaStream_t s) {
    if (a.T <= 0) return OK;
    const size_t items = static_cast<size_t>(a.T) * (a.heads + a.kv_heads);
    dec::attn_prep_kernel<<<nblk(items * 8, 256), 256, 8 * 4 * a.hd * sizeof(float), s>>>(a);
    DEC_LAUNCHED();
}
int dec_attention(const dec::AttnArgs& a, int n_tiles, int hd, cudaStream_t s) {
    if (n_tiles <= 0) return OK;
    const int tc = dec_attention_tc(a, n_tiles, hd, s);   // tcgen05 where it applies (head_dim 128)
    if (tc != ERR_NOT_SUPPORTED) return tc;
    const dim3 grid(n_tiles, a.heads);
    if (hd == 128) {
        const int smem = 3 * dec::T64 * (128 + 8) * 2;
        LAYA_CUDA(cudaFuncSetAttribute(dec::attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        dec::attention_kernel<128><<<grid, 128, smem, s>>>(a);
    } else if (hd == 64) {
        dec::attention_kernel<64><<<grid, 128, 3 * dec::T64 * (64 + 8) * 2, s>>>(a);
    } else if (hd == 32) {
        dec::attention_kernel<32><<<grid, 128, 3 * dec::T64 * (32 + 8) * 2, s>>>(a);
    } else {
        set_error("decoder attention: head_dim must be 32, 64 or 128");
        return ERR_NOT_SUPPORTED;
    }
    DEC_LAUNCHED();
}
int dec_gather_rows(const float* src, int ld_src, const int32_t* map, int rows, int n, float* dst, int ld_dst,
                    cudaStream_t s) {
    if (rows <= 0 || n <= 0) return OK;
    dec::gather_rows_kernel<<<nblk(static_cast<size_t>(rows) * n, 256), 256, 0, s>>>(src, ld_src, map, rows, n, dst, ld_dst);
    DEC_LAUNCHED();
}
int dec_add(float* x, const float* y, size_t n, cudaStream_t s) {
    if (n == 0) return OK;
    dec::add_kernel<<<nblk(n, 256), 256, 0, s>>>(x, y, n);
    DEC_LAUNCHED();
}
int dec_q8_logits(const dec::LogitArgs& a, cudaStream_t s) {
    if (a.n_seq <= 0 || a.n_labels <= 0) return OK;
    dec::q8_logits_kernel<<<nblk(static_cast<size_t>(a.n_seq) * a.n_labels * 32, 256), 256, 0, s>>>(a);
    DEC_LAUNCHED();
}

}  // namespace laya
