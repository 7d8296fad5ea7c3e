/*
 * laya_vnni.c — AVX-512 restatements of the reference's CPU product kernels, for the timed CPU baseline only.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): bench.py's cpu_baseline leg and its --impl reference arm time
 * the reference's algorithm on the GPU host's cores with these, so that the CPU figure is the reference's kernel
 * strength rather than a scalar restatement's.  Results are bit-identical to the scalar definitions in
 * laya_oracle.c (tests/test_oracle_vnni.py checks that), which stay the parity checker.
 *
 *   lv_q8_*      PackedMatrixQ8_0.Panel512 (Base/Numerics/PackedMatrixQ8_0.cs:329-525): weights packed in panels of
 *                64 columns, 4 consecutive codes of one column per int32 lane; activations offset to unsigned
 *                (q + 128) so vpdpbusd (u8 × s8 → s32, 4 products per lane) applies; each block's accumulator starts
 *                at −128·Σw of that column and block, which makes the block sum the exact Σ q_x·q_w; then
 *                acc = fma((float)Σ, d_w·d_x, acc) per block in increasing k, 3 rows × 64 columns at a time.
 *   lv_f32_*     PackedMatrix.Multiply (Base/Numerics/PackedMatrix.cs:204-305): weights packed in panels of 64
 *                columns, k-major; acc starts at the bias and takes one fma per input feature in increasing k,
 *                4 rows × 64 columns at a time.
 *   lv_attention AttentionKernels.Scores / WeightedSum (Base/Numerics/AttentionKernels.cs:30-127): keys transposed
 *                so 16 keys' scores accumulate side by side (one fma per head dimension in increasing d), the
 *                row's softmax, then the weighted sum of values 16 dimensions at a time (one fma per key in
 *                increasing key order); the same order as lo_attention, so the same bits.
 * Compiled with -mavx512f -mavx512bw -mavx512vnni -ffp-contract=off (only the explicit fmas fuse); callers check
 * lv_supported() first.
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define LV_PANEL 64
#define LV_BLOCK 32

int lv_supported(void)
{
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
           __builtin_cpu_supports("avx512vnni");
}

/* Bytes of the packed Q8_0 weight: codes, scales and negated column sums per (panel, block). */
long lv_q8_packed_bytes(int N, int K)
{
    long panels = (N + LV_PANEL - 1) / LV_PANEL, blocks = K / LV_BLOCK;
    return panels * blocks * (LV_PANEL * LV_BLOCK + LV_PANEL * 4 + LV_PANEL * 4);
}

/* codes [panel][block][group of 4 k][64 columns][4], then scales [panel][block][64] fp32 and −128·Σw
 * [panel][block][64] int32; columns past N are zero. */
void lv_q8_pack(const int8_t *qw, const float *dw, int N, int K, void *packed)
{
    const int panels = (N + LV_PANEL - 1) / LV_PANEL, blocks = K / LV_BLOCK;
    int8_t *codes = (int8_t *)packed;
    float *scales = (float *)(codes + (long)panels * blocks * LV_PANEL * LV_BLOCK);
    int32_t *negsum = (int32_t *)(scales + (long)panels * blocks * LV_PANEL);
    memset(packed, 0, lv_q8_packed_bytes(N, K));
    #pragma omp parallel for schedule(static)
    for (int p = 0; p < panels; ++p)
        for (int b = 0; b < blocks; ++b) {
            int8_t *cb = codes + ((long)p * blocks + b) * LV_PANEL * LV_BLOCK;
            for (int c = 0; c < LV_PANEL; ++c) {
                const int n = p * LV_PANEL + c;
                if (n >= N) continue;
                int32_t s = 0;
                for (int t = 0; t < LV_BLOCK; ++t) {
                    const int8_t v = qw[(long)n * K + b * LV_BLOCK + t];
                    cb[(t / 4) * LV_PANEL * 4 + c * 4 + (t % 4)] = v;
                    s += v;
                }
                scales[((long)p * blocks + b) * LV_PANEL + c] = dw[(long)n * blocks + b];
                negsum[((long)p * blocks + b) * LV_PANEL + c] = -128 * s;
            }
        }
}

static void lv_q8_panel(const uint8_t *xu, const float *dx, int rows, int K, const int8_t *codes, const float *scales,
                        const int32_t *negsum, int blocks, const float *bias, int n0, int N, float *out, int ldo)
{
    __m512 f[3][4];
    for (int c = 0; c < 4; ++c) {
        __m512 s = _mm512_setzero_ps();
        if (bias) {
            float tmp[16];
            for (int j = 0; j < 16; ++j) tmp[j] = (n0 + 16 * c + j < N) ? bias[n0 + 16 * c + j] : 0.0f;
            s = _mm512_loadu_ps(tmp);
        }
        for (int r = 0; r < 3; ++r) f[r][c] = s;
    }
    for (int b = 0; b < blocks; ++b) {
        const int32_t *z = negsum + (long)b * LV_PANEL;
        __m512i acc[3][4];
        for (int c = 0; c < 4; ++c) {
            const __m512i zc = _mm512_loadu_si512((const void *)(z + 16 * c));
            for (int r = 0; r < 3; ++r) acc[r][c] = zc;
        }
        const int8_t *cb = codes + (long)b * LV_PANEL * LV_BLOCK;
        for (int g = 0; g < LV_BLOCK / 4; ++g) {
            const __m512i w0 = _mm512_loadu_si512((const void *)(cb + g * 256));
            const __m512i w1 = _mm512_loadu_si512((const void *)(cb + g * 256 + 64));
            const __m512i w2 = _mm512_loadu_si512((const void *)(cb + g * 256 + 128));
            const __m512i w3 = _mm512_loadu_si512((const void *)(cb + g * 256 + 192));
            for (int r = 0; r < rows; ++r) {
                int32_t four;
                memcpy(&four, xu + (long)r * K + b * LV_BLOCK + 4 * g, 4);
                const __m512i x = _mm512_set1_epi32(four);
                acc[r][0] = _mm512_dpbusd_epi32(acc[r][0], x, w0);
                acc[r][1] = _mm512_dpbusd_epi32(acc[r][1], x, w1);
                acc[r][2] = _mm512_dpbusd_epi32(acc[r][2], x, w2);
                acc[r][3] = _mm512_dpbusd_epi32(acc[r][3], x, w3);
            }
        }
        const float *sc = scales + (long)b * LV_PANEL;
        for (int r = 0; r < rows; ++r) {
            const __m512 d = _mm512_set1_ps(dx[(long)r * blocks + b]);
            for (int c = 0; c < 4; ++c) {
                const __m512 dwdx = _mm512_mul_ps(_mm512_loadu_ps(sc + 16 * c), d);
                f[r][c] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(acc[r][c]), dwdx, f[r][c]);
            }
        }
    }
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < 4; ++c) {
            float tmp[16];
            _mm512_storeu_ps(tmp, f[r][c]);
            for (int j = 0; j < 16; ++j)
                if (n0 + 16 * c + j < N) out[(long)r * ldo + n0 + 16 * c + j] = tmp[j];
        }
}

/* out [rows, ldo] = Q8_0(qx, dx) · packed weight (+ bias); qx int8 [rows, K], dx fp32 [rows, K/32]. */
void lv_q8_matmul(const int8_t *qx, const float *dx, int rows, const void *packed, int N, int K, const float *bias,
                  float *out, int ldo, uint8_t *xu_scratch)
{
    const int panels = (N + LV_PANEL - 1) / LV_PANEL, blocks = K / LV_BLOCK;
    const int8_t *codes = (const int8_t *)packed;
    const float *scales = (const float *)(codes + (long)panels * blocks * LV_PANEL * LV_BLOCK);
    const int32_t *negsum = (const int32_t *)(scales + (long)panels * blocks * LV_PANEL);
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)rows * K; ++i) xu_scratch[i] = (uint8_t)(qx[i] + 128);
    const int rgroups = (rows + 2) / 3;
    #pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int p = 0; p < panels; ++p)
        for (int rg = 0; rg < rgroups; ++rg) {
            const int r0 = rg * 3, nr = rows - r0 < 3 ? rows - r0 : 3;
            lv_q8_panel(xu_scratch + (long)r0 * K, dx + (long)r0 * blocks, nr, K,
                        codes + (long)p * blocks * LV_PANEL * LV_BLOCK, scales + (long)p * blocks * LV_PANEL,
                        negsum + (long)p * blocks * LV_PANEL, blocks, bias, p * LV_PANEL, N, out + (long)r0 * ldo, ldo);
        }
}

/* ------------------------------------------------------------------------------------------------ fp32 */
long lv_f32_packed_floats(int N, int K) { return (long)((N + LV_PANEL - 1) / LV_PANEL) * K * LV_PANEL; }

/* w [N, K] -> [panel][k][64 columns], columns past N zero. */
void lv_f32_pack(const float *w, int N, int K, float *packed)
{
    const int panels = (N + LV_PANEL - 1) / LV_PANEL;
    #pragma omp parallel for schedule(static)
    for (int p = 0; p < panels; ++p)
        for (int k = 0; k < K; ++k)
            for (int c = 0; c < LV_PANEL; ++c) {
                const int n = p * LV_PANEL + c;
                packed[((long)p * K + k) * LV_PANEL + c] = n < N ? w[(long)n * K + k] : 0.0f;
            }
}

void lv_linear_f32(const float *x, int rows, int ldx, const float *packed, int N, int K, const float *bias, float *out,
                   int ldo)
{
    const int panels = (N + LV_PANEL - 1) / LV_PANEL, rgroups = (rows + 3) / 4;
    #pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int p = 0; p < panels; ++p)
        for (int rg = 0; rg < rgroups; ++rg) {
            const int r0 = rg * 4, nr = rows - r0 < 4 ? rows - r0 : 4, n0 = p * LV_PANEL;
            __m512 f[4][4];
            for (int c = 0; c < 4; ++c) {
                __m512 s = _mm512_setzero_ps();
                if (bias) {
                    float tmp[16];
                    for (int j = 0; j < 16; ++j) tmp[j] = (n0 + 16 * c + j < N) ? bias[n0 + 16 * c + j] : 0.0f;
                    s = _mm512_loadu_ps(tmp);
                }
                for (int r = 0; r < 4; ++r) f[r][c] = s;
            }
            const float *wp = packed + (long)p * K * LV_PANEL;
            for (int k = 0; k < K; ++k) {
                const __m512 w0 = _mm512_loadu_ps(wp + (long)k * LV_PANEL), w1 = _mm512_loadu_ps(wp + (long)k * LV_PANEL + 16),
                             w2 = _mm512_loadu_ps(wp + (long)k * LV_PANEL + 32), w3 = _mm512_loadu_ps(wp + (long)k * LV_PANEL + 48);
                for (int r = 0; r < nr; ++r) {
                    const __m512 xv = _mm512_set1_ps(x[(long)(r0 + r) * ldx + k]);
                    f[r][0] = _mm512_fmadd_ps(xv, w0, f[r][0]);
                    f[r][1] = _mm512_fmadd_ps(xv, w1, f[r][1]);
                    f[r][2] = _mm512_fmadd_ps(xv, w2, f[r][2]);
                    f[r][3] = _mm512_fmadd_ps(xv, w3, f[r][3]);
                }
            }
            for (int r = 0; r < nr; ++r)
                for (int c = 0; c < 4; ++c) {
                    float tmp[16];
                    _mm512_storeu_ps(tmp, f[r][c]);
                    for (int j = 0; j < 16; ++j)
                        if (n0 + 16 * c + j < N) out[(long)(r0 + r) * ldo + n0 + 16 * c + j] = tmp[j];
                }
        }
}

/* ------------------------------------------------------------------------------------------------ attention */
/* lo_softmax (laya_oracle.c), restated unchanged: max, exp(v − max) with libm's expf summed in order, scale. */
static void lv_softmax(float *v, int n)
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

static void lv_rope(float *v, int head_dim, const float *cosp, const float *sinp)
{
    int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        float a = v[i], b = v[i + half];
        v[i] = a * cosp[i] - b * sinp[i];
        v[i + half] = b * cosp[i] + a * sinp[i];
    }
}

/* lo_attention's contract (qkv [T, 3·hidden], segments, ±window or global, rotary tables or none) for head_dim a
 * multiple of 16. */
void lv_attention(const float *qkv, int hidden, int heads, const int *seg_start, const int *seg_len, int nseg,
                  int window, const float *cosv, const float *sinv, float *out)
{
    const int hd = hidden / heads, stride = 3 * hidden, half = hd / 2;
    const float scale = 1.0f / sqrtf((float)hd);
    #pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int s = 0; s < nseg; ++s)
        for (int h = 0; h < heads; ++h) {
            const int L = seg_len[s], start = seg_start[s];
            if (L <= 0) continue;
            const int Lp = (L + 15) / 16 * 16;
            float *q = (float *)malloc(sizeof(float) * (size_t)L * hd);
            float *kt = (float *)calloc((size_t)hd * Lp, sizeof(float));   /* [d][key] */
            float *v = (float *)malloc(sizeof(float) * (size_t)L * hd);
            float *sc = (float *)malloc(sizeof(float) * (size_t)Lp);
            float *kr = (float *)malloc(sizeof(float) * (size_t)hd);
            for (int t = 0; t < L; ++t) {
                const float *row = qkv + (long)(start + t) * stride;
                memcpy(q + (long)t * hd, row + h * hd, sizeof(float) * hd);
                memcpy(kr, row + hidden + h * hd, sizeof(float) * hd);
                memcpy(v + (long)t * hd, row + 2 * hidden + h * hd, sizeof(float) * hd);
                if (cosv) {
                    lv_rope(q + (long)t * hd, hd, cosv + (long)t * half, sinv + (long)t * half);
                    lv_rope(kr, hd, cosv + (long)t * half, sinv + (long)t * half);
                }
                for (int d = 0; d < hd; ++d) kt[(long)d * Lp + t] = kr[d];
            }
            const __m512 vscale = _mm512_set1_ps(scale);
            for (int t = 0; t < L; ++t) {
                const int first = window < 0 ? 0 : (t - window > 0 ? t - window : 0);
                const int last = window < 0 ? L - 1 : (t + window < L - 1 ? t + window : L - 1);
                const int count = last - first + 1;
                const float *qt = q + (long)t * hd;
                for (int j = 0; j < count; j += 16) {
                    __m512 acc = _mm512_setzero_ps();
                    for (int d = 0; d < hd; ++d)
                        acc = _mm512_fmadd_ps(_mm512_set1_ps(qt[d]), _mm512_loadu_ps(kt + (long)d * Lp + first + j), acc);
                    float tmp[16];
                    _mm512_storeu_ps(tmp, _mm512_mul_ps(acc, vscale));
                    for (int e = 0; e < 16 && j + e < count; ++e) sc[j + e] = tmp[e];
                }
                lv_softmax(sc, count);
                float *o = out + (long)(start + t) * hidden + h * hd;
                for (int d0 = 0; d0 < hd; d0 += 16) {
                    __m512 acc = _mm512_setzero_ps();
                    for (int j = 0; j < count; ++j)
                        acc = _mm512_fmadd_ps(_mm512_set1_ps(sc[j]), _mm512_loadu_ps(v + (long)(first + j) * hd + d0), acc);
                    _mm512_storeu_ps(o + d0, acc);
                }
            }
            free(q); free(kt); free(v); free(sc); free(kr);
        }
}
