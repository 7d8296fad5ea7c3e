/*
 * laya_oracle.c — CPU restatement of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (laya_b200/) links, loads or calls this file.  It is
 * the checker the parity tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg compare the CUDA
 * library against.  Parity is pinned: the tests check this code against the reference's own golden
 * vectors (Q8_0 known answers, the qwen35-tiny `matmul.*` tensors, the training-tiny logits and
 * gradients), see tests/test_oracle.py.
 *
 * Every function follows one reference routine, cited by file:line inside the reference project
 * (theolivenbaum/laya).  Floating-point operations are written in the reference's order: explicit fmaf()
 * where the reference calls FusedMultiplyAdd, plain multiply-then-add elsewhere (the .NET JIT does not
 * contract), and the file is compiled with -ffp-contract=off so the compiler cannot fuse on its own.
 *
 * Vector<float> in the reference is 256 bits wide on x86 (8 lanes): reductions that the reference runs
 * lane-parallel (Sum, Dot, LayerNorm's variance) are restated with 8 lane accumulators.  The horizontal
 * reduction order of .NET's Vector.Sum is not documented; it is restated here as (lo+hi) then pairwise,
 * which is an ulp-level choice — parity for those stages is tolerance-based.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define LO_W 8         /* Vector<float>.Count of the reference on x86 */
#define LO_BLOCK 32    /* Q8_0 block size (PackedMatrixQ8_0.cs:17) */

int lo_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void lo_set_num_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------------------------------ */
/* fp16 rounding of a float (C# (float)(Half)x): round to nearest even, with subnormals and overflow. */
static float lo_round_fp16(float x)
{
    uint32_t u;
    memcpy(&u, &x, 4);
    uint32_t sign = u & 0x80000000u;
    uint32_t absu = u & 0x7fffffffu;
    float ax;
    memcpy(&ax, &absu, 4);
    if (absu >= 0x7f800000u) return x;                    /* inf / nan */
    if (ax >= 65520.0f) {                                 /* rounds to inf */
        uint32_t r = sign | 0x7f800000u; float f; memcpy(&f, &r, 4); return f;
    }
    float r;
    if (ax < 6.103515625e-05f) {                          /* fp16 subnormal range: quantum 2^-24 */
        const float q = 5.9604644775390625e-08f;
        r = nearbyintf(ax / q) * q;                       /* ax/q exact (power of two), RNE via nearbyintf */
    } else {
        /* keep 11 significant bits: RNE on the low 13 mantissa bits */
        uint32_t lsb = (absu >> 13) & 1u;
        uint32_t rounded = absu + 0x0fffu + lsb;
        rounded &= ~0x1fffu;
        memcpy(&r, &rounded, 4);
    }
    uint32_t ru; memcpy(&ru, &r, 4); ru |= sign; memcpy(&r, &ru, 4);
    return r;
}

float lo_fp16_round(float x) { return lo_round_fp16(x); }

/* ------------------------------------------------------------------------------------------------ */
/* Q8_0 (PackedMatrixQ8_0.cs:15-72) */

/* Q8_0.QuantizeWeightBlock (PackedMatrixQ8_0.cs:20-28): d = amax/127, id = 1/d, round half away. */
float lo_q8_quantize_weight_block(const float *x, int8_t *q)
{
    float amax = 0.0f;
    for (int j = 0; j < LO_BLOCK; ++j) amax = fmaxf(amax, fabsf(x[j]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < LO_BLOCK; ++j) q[j] = (int8_t)roundf(x[j] * id);
    return lo_round_fp16(d);
}

/* Every block of a PyTorch [N, K] weight; d is [N, K/32] (the packed layout's values, PackedMatrixQ8_0.cs:187-206). */
void lo_q8_quantize_weights(const float *w, int N, int K, int8_t *q, float *d)
{
    int blocks = K / LO_BLOCK;
    #pragma omp parallel for schedule(static)
    for (int c = 0; c < N; ++c)
        for (int b = 0; b < blocks; ++b)
            d[(long)c * blocks + b] = lo_q8_quantize_weight_block(w + (long)c * K + b * LO_BLOCK,
                                                                 q + (long)c * K + b * LO_BLOCK);
}

/*
 * Q8_0.QuantizeActivations (PackedMatrixQ8_0.cs:35-71): amax, d = amax/127 stored fp16, id = 127/amax,
 * q = round-half-even(x * id).  The reference stores q+128 as bytes for vpdpbusd; this stores q itself
 * (int8), the same information.  q is [rows, K] packed, d is [rows, K/32].
 */
void lo_q8_quantize_activations(const float *in, int rows, int stride, int K, int8_t *q, float *d)
{
    int blocks = K / LO_BLOCK;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *src = in + (long)r * stride;
        for (int b = 0; b < blocks; ++b) {
            const float *x = src + b * LO_BLOCK;
            float amax = 0.0f;
            for (int j = 0; j < LO_BLOCK; ++j) amax = fmaxf(amax, fabsf(x[j]));
            float dd = amax / 127.0f;
            float id = amax != 0.0f ? 127.0f / amax : 0.0f;
            for (int j = 0; j < LO_BLOCK; ++j) q[(long)r * K + b * LO_BLOCK + j] = (int8_t)(int)nearbyintf(x[j] * id);
            d[(long)r * blocks + b] = lo_round_fp16(dd);
        }
    }
}

/*
 * The Q8_0 product by its definition (PackedMatrixQ8_0Tests.cs:145-182, the bit-exact reference every
 * kernel of PackedMatrixQ8_0.cs:329-557 must equal): per block an exact int32 dot, then
 * acc = fma((float)sum, d_w * d_x, acc), blocks in increasing k, acc starting at the bias.
 */
void lo_q8_matmul(const int8_t *qx, const float *dx, int rows, const int8_t *qw, const float *dw, int N, int K,
                  const float *bias, float *out, int ldo)
{
    int blocks = K / LO_BLOCK;
    #pragma omp parallel for schedule(dynamic, 1)
    for (int r = 0; r < rows; ++r) {
        const int8_t *xr = qx + (long)r * K;
        const float *dxr = dx + (long)r * blocks;
        for (int c = 0; c < N; ++c) {
            const int8_t *wc = qw + (long)c * K;
            const float *dwc = dw + (long)c * blocks;
            float acc = bias ? bias[c] : 0.0f;
            for (int b = 0; b < blocks; ++b) {
                int32_t sum = 0;
                const int8_t *xa = xr + b * LO_BLOCK, *wa = wc + b * LO_BLOCK;
                for (int t = 0; t < LO_BLOCK; ++t) sum += (int32_t)xa[t] * (int32_t)wa[t];
                acc = fmaf((float)sum, dwc[b] * dxr[b], acc);
            }
            out[(long)r * ldo + c] = acc;
        }
    }
}

/* Exact int32 block dots, [rows, N, K/32]: what the bit-exact check of the tensor-core path compares. */
void lo_q8_block_dots(const int8_t *qx, int rows, const int8_t *qw, int N, int K, int32_t *dots)
{
    int blocks = K / LO_BLOCK;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < N; ++c)
            for (int b = 0; b < blocks; ++b) {
                int32_t sum = 0;
                for (int t = 0; t < LO_BLOCK; ++t)
                    sum += (int32_t)qx[(long)r * K + b * LO_BLOCK + t] * (int32_t)qw[(long)c * K + b * LO_BLOCK + t];
                dots[((long)r * N + c) * blocks + b] = sum;
            }
}

/* ------------------------------------------------------------------------------------------------ */
/* fp32 linear, PackedMatrix.Multiply (PackedMatrix.cs:121-305): acc starts at the bias and takes one
 * fma per input feature in increasing order; out = x · Wᵀ + b. */
void lo_linear_f32(const float *x, int rows, int ldx, const float *w, int N, int K, const float *bias,
                   float *out, int ldo)
{
    #pragma omp parallel for schedule(dynamic, 4)
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < N; ++c) {
            float acc = bias ? bias[c] : 0.0f;
            const float *xr = x + (long)r * ldx, *wc = w + (long)c * K;
            for (int k = 0; k < K; ++k) acc = fmaf(xr[k], wc[k], acc);
            out[(long)r * ldo + c] = acc;
        }
}

/* ------------------------------------------------------------------------------------------------ */
/* SimdOps (SimdOps.cs) */

static float lo_hsum(const float *acc)
{
    float lo[4];
    for (int i = 0; i < 4; ++i) lo[i] = acc[i] + acc[i + 4];
    return (lo[0] + lo[1]) + (lo[2] + lo[3]);
}

/* SimdOps.Sum (SimdOps.cs:~190): lane accumulators, horizontal sum, scalar tail. */
float lo_sum(const float *v, int n)
{
    float acc[LO_W] = {0};
    int i = 0;
    for (; i <= n - LO_W; i += LO_W)
        for (int l = 0; l < LO_W; ++l) acc[l] += v[i + l];
    float s = lo_hsum(acc);
    for (; i < n; ++i) s += v[i];
    return s;
}

/* SimdOps.Dot (SimdOps.cs:64-85): two lane accumulators with FMA, then scalar tail (multiply, add). */
float lo_dot(const float *a, const float *b, int n)
{
    float s0[LO_W] = {0}, s1[LO_W] = {0};
    int i = 0;
    for (; i <= n - 2 * LO_W; i += 2 * LO_W)
        for (int l = 0; l < LO_W; ++l) {
            s0[l] = fmaf(a[i + l], b[i + l], s0[l]);
            s1[l] = fmaf(a[i + LO_W + l], b[i + LO_W + l], s1[l]);
        }
    for (; i <= n - LO_W; i += LO_W)
        for (int l = 0; l < LO_W; ++l) s0[l] = fmaf(a[i + l], b[i + l], s0[l]);
    float sum = lo_hsum(s0) + lo_hsum(s1);
    for (; i < n; ++i) sum += a[i] * b[i];
    return sum;
}

/* SimdOps.LayerNorm (SimdOps.cs:234-272): mean by Sum, biased variance by lane FMA, eps inside sqrt. */
static void lo_layer_norm_row(const float *in, int n, const float *w, const float *bias, float eps, float *out)
{
    float mean = lo_sum(in, n) / (float)n;
    float acc[LO_W] = {0};
    int i = 0;
    for (; i <= n - LO_W; i += LO_W)
        for (int l = 0; l < LO_W; ++l) { float d = in[i + l] - mean; acc[l] = fmaf(d, d, acc[l]); }
    float var = lo_hsum(acc);
    for (; i < n; ++i) { float d = in[i] - mean; var += d * d; }
    var /= (float)n;
    float inv = 1.0f / sqrtf(var + eps);
    for (i = 0; i < n; ++i) {
        float v = (in[i] - mean) * inv * w[i];
        out[i] = bias ? v + bias[i] : v;
    }
}

void lo_layer_norm_rows(const float *in, int rows, int n, const float *w, const float *bias, float eps, float *out)
{
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) lo_layer_norm_row(in + (long)r * n, n, w, bias, eps, out + (long)r * n);
}

/* SimdOps.Exp (SimdOps.cs:368-390): 2^n · Taylor-6(r) with a two-constant ln2 reduction. */
float lo_exp_vec(float value)
{
    float x = fminf(fmaxf(value, -87.3f), 88.7f);
    float n = floorf(fmaf(x, 1.4426950408889634f, 0.5f));
    float r = fmaf(n, -0.693359375f, x);
    r = fmaf(n, 2.12194440e-4f, r);
    float p = 1.0f / 720.0f;
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int32_t e = ((int32_t)n + 127) << 23;
    float scale; memcpy(&scale, &e, 4);
    return p * scale;
}

/* SimdOps.Erf(Vector<float>) (SimdOps.cs:329-356): Numerical Recipes erfc rational form in float. */
float lo_erf_vec(float value)
{
    float sign = value < 0.0f ? -1.0f : 1.0f;
    float ax = fabsf(value);
    float t = 1.0f / (1.0f + 0.5f * ax);
    float poly = 0.17087277f;
    poly = fmaf(poly, t, -0.82215223f);
    poly = fmaf(poly, t, 1.48851587f);
    poly = fmaf(poly, t, -1.13520398f);
    poly = fmaf(poly, t, 0.27886807f);
    poly = fmaf(poly, t, -0.18628806f);
    poly = fmaf(poly, t, 0.09678418f);
    poly = fmaf(poly, t, 0.37409196f);
    poly = fmaf(poly, t, 1.00002368f);
    poly = fmaf(poly, t, -1.26551223f);
    poly -= ax * ax;
    float y = t * lo_exp_vec(poly);
    return sign * (ax > 6.0f ? 1.0f : 1.0f - y);
}

/* SimdOps.Gelu (SimdOps.cs:305-323): x * 0.5 * (1 + erf(x / sqrt 2)), vector path. */
float lo_gelu1(float x) { return x * 0.5f * (1.0f + lo_erf_vec(x * 0.70710678118654752f)); }

void lo_gelu(float *v, long n)
{
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) v[i] = lo_gelu1(v[i]);
}

/* SimdOps.Relu (SimdOps.cs:393-403) */
void lo_relu(float *v, long n)
{
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) v[i] = fmaxf(v[i], 0.0f);
}

/* SimdOps.Softmax (SimdOps.cs:275-291): max subtraction, MathF.Exp, scale by 1/total. */
void lo_softmax(float *v, int n)
{
    if (n <= 0) return;
    float mx = v[0];
    for (int i = 1; i < n; ++i) mx = fmaxf(mx, v[i]);
    if (isinf(mx) && mx < 0) { memset(v, 0, sizeof(float) * n); return; }
    float total = 0.0f;
    for (int i = 0; i < n; ++i) { float e = expf(v[i] - mx); v[i] = e; total += e; }
    float s = total > 0.0f ? 1.0f / total : 0.0f;
    for (int i = 0; i < n; ++i) v[i] *= s;
}

/* ModernBertEncoder.GeGlu (ModernBertEncoder.cs:204-214): gelu(wide[:, :I]) * wide[:, I:]. */
void lo_geglu(const float *wide, int rows, int I, float *out)
{
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < rows; ++t)
        for (int i = 0; i < I; ++i) {
            float g = lo_gelu1(wide[(long)t * 2 * I + i]);
            out[(long)t * I + i] = g * wide[(long)t * 2 * I + I + i];
        }
}

/* RopeCache (ModernBertEncoder.cs:341-379): cos/sin [positions, head_dim/2], angles in double. */
void lo_rope_table(int head_dim, double theta, int positions, float *cosv, float *sinv)
{
    int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        double inv = 1.0 / pow(theta, 2.0 * i / head_dim);
        for (int p = 0; p < positions; ++p) {
            double a = p * inv;
            cosv[p * half + i] = (float)cos(a);
            sinv[p * half + i] = (float)sin(a);
        }
    }
}

/* RopeCache.Apply (ModernBertEncoder.cs:386-400): rotate-half convention. */
static void lo_rope_apply(float *v, int head_dim, const float *cosp, const float *sinp)
{
    int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        float a = v[i], b = v[i + half];
        v[i] = a * cosp[i] - b * sinp[i];
        v[i + half] = b * cosp[i] + a * sinp[i];
    }
}

/*
 * Multi-head attention per (segment, head) over a packed [T, 3*hidden] qkv buffer
 * (ModernBertEncoder.Attention, ModernBertEncoder.cs:230-302, with AttentionKernels.Scores/WeightedSum,
 * AttentionKernels.cs:30-125; DecisionModel.HeadAttention, DecisionModel.cs:319-368, is the same with
 * no rotary and no window).  window < 0 means global; otherwise keys in [t-window, t+window].
 * Positions restart at 0 in every segment.  cos/sin may be NULL (no rotary).
 */
void lo_attention(const float *qkv, int hidden, int heads, const int *seg_start, const int *seg_len, int nseg,
                  int window, const float *cosv, const float *sinv, float *out)
{
    int head_dim = hidden / heads;
    int stride = 3 * hidden;
    float scale = 1.0f / sqrtf((float)head_dim);
    int half = head_dim / 2;
    #pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int s = 0; s < nseg; ++s)
        for (int h = 0; h < heads; ++h) {
            int L = seg_len[s], start = seg_start[s];
            if (L <= 0) continue;
            float *q = (float *)malloc(sizeof(float) * (size_t)L * head_dim);
            float *k = (float *)malloc(sizeof(float) * (size_t)L * head_dim);
            float *v = (float *)malloc(sizeof(float) * (size_t)L * head_dim);
            float *sc = (float *)malloc(sizeof(float) * (size_t)L);
            for (int t = 0; t < L; ++t) {
                const float *row = qkv + (long)(start + t) * stride;
                memcpy(q + (long)t * head_dim, row + h * head_dim, sizeof(float) * head_dim);
                memcpy(k + (long)t * head_dim, row + hidden + h * head_dim, sizeof(float) * head_dim);
                memcpy(v + (long)t * head_dim, row + 2 * hidden + h * head_dim, sizeof(float) * head_dim);
                if (cosv) {
                    lo_rope_apply(q + (long)t * head_dim, head_dim, cosv + (long)t * half, sinv + (long)t * half);
                    lo_rope_apply(k + (long)t * head_dim, head_dim, cosv + (long)t * half, sinv + (long)t * half);
                }
            }
            for (int t = 0; t < L; ++t) {
                int first = window < 0 ? 0 : (t - window > 0 ? t - window : 0);
                int last = window < 0 ? L - 1 : (t + window < L - 1 ? t + window : L - 1);
                int count = last - first + 1;
                const float *qt = q + (long)t * head_dim;
                for (int j = 0; j < count; ++j) {
                    const float *kj = k + (long)(first + j) * head_dim;
                    float acc = 0.0f;
                    for (int d = 0; d < head_dim; ++d) acc = fmaf(qt[d], kj[d], acc);
                    sc[j] = acc * scale;
                }
                lo_softmax(sc, count);
                float *o = out + (long)(start + t) * hidden + h * head_dim;
                for (int d = 0; d < head_dim; ++d) {
                    float acc = 0.0f;
                    for (int j = 0; j < count; ++j) acc = fmaf(sc[j], v[(long)(first + j) * head_dim + d], acc);
                    o[d] = acc;
                }
            }
            free(q); free(k); free(v); free(sc);
        }
}

/* SimdOps.Add (SimdOps.cs:88-97): dst += src. */
void lo_add(float *dst, const float *src, long n)
{
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) dst[i] += src[i];
}

/* ------------------------------------------------------------------------------------------------ */
/* The Qwen3.5 decoder behind Mica (DecoderKernels.cs, Qwen35Model.cs) */

/* DecoderKernels.SumOfSquares (DecoderKernels.cs:15-28): lane accumulators by FMA, Vector.Sum, scalar tail. */
static float lo_sum_squares(const float *v, int n)
{
    float acc[LO_W] = {0};
    int i = 0;
    for (; i <= n - LO_W; i += LO_W)
        for (int l = 0; l < LO_W; ++l) acc[l] = fmaf(v[i + l], v[i + l], acc[l]);
    float s = lo_hsum(acc);
    for (; i < n; ++i) s += v[i] * v[i];
    return s;
}

/* DecoderKernels.RmsNorm (DecoderKernels.cs:34-46): x · (1 / sqrt(Σx²/n + eps)) · scale, scale = 1 + weight. */
void lo_rms_norm_rows(const float *in, int rows, int n, const float *scale, float eps, float *out)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *x = in + (long)r * n;
        float *y = out + (long)r * n;
        float inv = 1.0f / sqrtf(lo_sum_squares(x, n) / (float)n + eps);
        for (int i = 0; i < n; ++i) y[i] = x[i] * inv * scale[i];
    }
}

/* DecoderKernels.Sigmoid / Silu on Vector<float> (DecoderKernels.cs:150-151): 1 / (1 + SimdOps.Exp(-x)). */
static float lo_sigmoid_vec(float x) { return 1.0f / (1.0f + lo_exp_vec(-x)); }

void lo_silu_vec(float *v, long n)
{
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) v[i] = v[i] * lo_sigmoid_vec(v[i]);
}

/* DecoderKernels.SiluMultiply (DecoderKernels.cs:97-107): silu(gate) · up, rows of width n in [gate | up] rows. */
void lo_silu_multiply(const float *gate_up, int rows, int n, float *out)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *g = gate_up + (long)r * 2 * n, *u = g + n;
        for (int i = 0; i < n; ++i) out[(long)r * n + i] = g[i] * lo_sigmoid_vec(g[i]) * u[i];
    }
}

/* DecoderKernels.MultiplySigmoid (DecoderKernels.cs:125-135): values · sigmoid(gate). */
void lo_multiply_sigmoid(float *v, const float *gate, long n)
{
    for (long i = 0; i < n; ++i) v[i] = v[i] * lo_sigmoid_vec(gate[i]);
}

/* DecoderKernels.L2Normalize (DecoderKernels.cs:67-85): x · (1 / sqrt(Σx² + eps)) (· extra). */
void lo_l2_normalize(float *v, int n, float eps, float extra)
{
    float inv = 1.0f / sqrtf(lo_sum_squares(v, n) + eps);
    for (int i = 0; i < n; ++i) {
        float x = v[i] * inv;
        v[i] = extra != 1.0f ? x * extra : x;
    }
}

/* DecoderKernels.RmsNormGated (DecoderKernels.cs:52-64): weight · (x · inv) · silu(gate). */
void lo_rms_norm_gated(const float *in, const float *gate, const float *weight, int n, float eps, float *out)
{
    float inv = 1.0f / sqrtf(lo_sum_squares(in, n) / (float)n + eps);
    for (int i = 0; i < n; ++i) {
        float g = gate[i];
        out[i] = weight[i] * (in[i] * inv) * (g * lo_sigmoid_vec(g));
    }
}

/* The gated delta rule of one value head (Qwen35Model.Recurrence, Qwen35Model.cs:924-972, the two-sweep form that
 * DecoderKernels.GatedDeltaRule128 reproduces bit for bit), on a row-major [dk, dv] state, per token:
 *   S ← S·g;  m = Sᵀk (FMA, i ascending);  δ = (v − m)·β;  S ← S + k ⊗ δ (FMA);  o = Sᵀq (FMA, i ascending). */
void lo_delta_rule(float *state, int dk, int dv, int rows, const float *q, const float *k, const float *v, int stride,
                   const float *decay, const float *beta, int gstride, float *out, int ostride)
{
    float *m = (float *)malloc(sizeof(float) * dv), *d = (float *)malloc(sizeof(float) * dv);
    for (int t = 0; t < rows; ++t) {
        const float *qt = q + (long)t * stride, *kt = k + (long)t * stride, *vt = v + (long)t * stride;
        const float g = decay[(long)t * gstride], b = beta[(long)t * gstride];
        float *ot = out + (long)t * ostride;
        for (int j = 0; j < dv; ++j) m[j] = 0.0f;
        for (int i = 0; i < dk; ++i) {
            float *s = state + (long)i * dv;
            for (int j = 0; j < dv; ++j) {
                s[j] = s[j] * g;
                m[j] = fmaf(s[j], kt[i], m[j]);
            }
        }
        for (int j = 0; j < dv; ++j) { d[j] = (vt[j] - m[j]) * b; ot[j] = 0.0f; }
        for (int i = 0; i < dk; ++i) {
            float *s = state + (long)i * dv;
            for (int j = 0; j < dv; ++j) {
                s[j] = fmaf(d[j], kt[i], s[j]);
                ot[j] = fmaf(s[j], qt[i], ot[j]);
            }
        }
    }
    free(m);
    free(d);
}
