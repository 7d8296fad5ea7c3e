// train.h — argument blocks of the training-path kernels (internal to the library).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace laya {
namespace bf {
enum Epi : int {
    EPI_BF16 = 0,     // out bf16 = A·Bᵀ (+ bias)
    EPI_F32 = 1,      // out fp32 = A·Bᵀ (+ bias)
    EPI_F32_ADD = 2,  // out fp32 += A·Bᵀ (+ bias), by TMA reduce-add
    EPI_QKV = 3,      // attention input: (A·Bᵀ + bias) with columns < rot_cols rotated at each row's segment position
                      // (pairs (i, i + 32) of every 64-column head), out bf16 hi and out2 bf16 lo (or no lo)
};
// out[M, N] = A · Bᵀ with A [M, K] and B [N, K] in the logical view; a_mn / b_mn say the operand is stored with the
// M (N) index contiguous instead of K: A as [K, lda] and B as [K, ldb].  Row strides in elements.
// With A2 and B2 (the bf16 remainders x − bf16(x) of fp32 operands, same layout and strides as A and B) the product
// is A·Bᵀ + A2·Bᵀ + A·B2ᵀ: the three leading terms of (A + A2)(B + B2)ᵀ, accurate to about 2^-16 relative.  With A2
// alone (B exactly bf16, as a bf16 checkpoint's weights are) it is A·Bᵀ + A2·Bᵀ, to the same accuracy.
struct Args {
    int M, N, K;
    const __nv_bfloat16* A; int lda; int a_mn;
    const __nv_bfloat16* B; int ldb; int b_mn;
    const float* bias;
    int epi;
    void* out; int ldo;
    int* err;
    const __nv_bfloat16* A2 = nullptr;
    const __nv_bfloat16* B2 = nullptr;
    int ksplit_ok = 0;   // EPI_F32_ADD only: K may be split into chunks that reduce-add (summation order varies)
    // EPI_QKV (CTA-pair products only; ERR_NOT_SUPPORTED otherwise): the low parts, and the rotary tables
    // [position, 32] with each row's position = row − seg_start[tok_item[row]]; cosv null: no rotation
    void* out2 = nullptr;
    const int32_t* tok_item = nullptr; const int32_t* seg_start = nullptr;
    const float* cosv = nullptr; const float* sinv = nullptr; int rot_cols = 0;
};
int gemm(const Args& a, cudaStream_t stream);
}  // namespace bf
}  // namespace laya

namespace laya {

// ---- flash.cu
namespace fa {
struct Args {
    const __nv_bfloat16* qkv; int ld; int hidden; int heads;        // [T, ld] q | k | v at 0, hidden, 2·hidden; q, k rotated
    const int32_t* seg_start; const int32_t* seg_len;
    const int32_t* tile_item; const int32_t* tile_p0; const int32_t* n_tiles;   // 64-row tiles of every segment
    int window;                                                      // < 0: global
    float scale;                                                     // 1/sqrt(head_dim)
    const float* cosv; const float* sinv;                            // [positions, head_dim/2] or null: the backward's
                                                                     // inverse rotation of dq and dk
    float dropout; float keep; uint64_t seed;                        // dropout on the probabilities
    __nv_bfloat16* out; int ldo; float* lse;                         // context [T, ldo] bf16, row log-sum-exp [T, heads]
    const __nv_bfloat16* dout; float* dsum;                          // backward: d context [T, ldo], Σ dO·O [T, heads]
    __nv_bfloat16* dqkv; int lddq;                                   // backward output [T, lddq]
    const __nv_bfloat16* qkv_lo;                                     // accurate forward: low parts of qkv (else null)
    __nv_bfloat16* out_lo;                                           // accurate forward: context low part
    // the tcgen05 forward (head_dim 64): 128-row query tiles of every segment, and the token count
    const int32_t* tq_item; const int32_t* tq_p0; const int32_t* n_tq; int max_tq; int T;
    // the two-tile forward: 256-row pair tiles of every segment
    const int32_t* tp_item = nullptr; const int32_t* tp_p0 = nullptr; const int32_t* n_tp = nullptr; int max_tp = 0;
    int* err;
    // the backward's dS scratch (flash_tc.cu): the dK/dV kernel leaves each 128-key × 64-query dSᵀ tile there and dQ
    // = dS·K streams them back; tile (g, j, head) at 1 + (g·ds_nq + j)·heads + head (16 KB each, tile 0 zeros); null:
    // dQ recomputes S and dP
    uint8_t* ds = nullptr; int ds_nq = 0;
    // the dropout decisions of this layer's probabilities, precomputed by drop_mask (null: the kernels evaluate the
    // counter hash per probability): word (head h, row t, w) at dmask[(h·dmask_rows + t)·dmask_w + w], bit i set when
    // the probability of row t for key 32·w + i of its segment is kept; dmask_w is a multiple of 4 covering the
    // longest segment rounded up to 128 keys
    const uint32_t* dmask = nullptr; int dmask_w = 0; int dmask_rows = 0;
};
}  // namespace fa
// Fills `mask` (a.dmask_w words per row, a.dmask_rows rows per head) for rows [0, a.T) with the decisions the counter
// hash of Ops.Dropout makes for a.seed and a.dropout (flash_pp.cu).
int drop_mask(const fa::Args& a, const int32_t* tok_item, uint32_t* mask, cudaStream_t s);
// q, k rotated at their segment positions (cosv null: no rotation), v copied, from fp32 or bf16 [T, lds] into bf16
// hi [T, ldd] (+ lo parts when lo is set); in place when src == hi (bf16).
int attn_prep(const void* src, int src_f32, int lds, int T, int hidden, int heads, const int32_t* tok_item,
              const int32_t* seg_start, const float* cosv, const float* sinv, __nv_bfloat16* hi, __nv_bfloat16* lo,
              int ldd, cudaStream_t s);
int flash_forward(const fa::Args& a, int max_tiles, cudaStream_t s);
int flash_forward_tc(const fa::Args& a, cudaStream_t s);   // flash_tc.cu: head_dim 64 (ERR_NOT_SUPPORTED otherwise)
int flash_forward_pp(const fa::Args& a, cudaStream_t s);   // flash_pp.cu: head_dim 64, two query tiles per CTA
int flash_backward_dkdv_tc(const fa::Args& a, cudaStream_t s);   // flash_tc.cu: dK, dV for head_dim 64
int flash_backward_dq_tc(const fa::Args& a, cudaStream_t s);     // flash_tc.cu: dQ for head_dim 64
int flash_backward_dq_ds(const fa::Args& a, cudaStream_t s);     // flash_tc.cu: dQ = dS·K from the dS scratch
// The decision forward's attention (inference) on the tensor cores: qkv16 [T, ld] fp16 = rotated q | k | v, 128-row
// query tiles of every segment, context out as Q8_0 codes q [T, hidden] and scales d [hidden/32, ldd].
struct InferAttn {
    const __half* qkv16; int ld; int hidden, heads, T;
    const int32_t* seg_start; const int32_t* seg_len;
    const int32_t* tq_item; const int32_t* tq_p0; const int32_t* n_tq; int max_tq;
    int window; float scale;
    __half* q; float* d; int ldd;            // Q8_0 codes and scales, or (q null) ...
    __nv_bfloat16* hi; __nv_bfloat16* lo;     // ... the context as bf16 hi/lo parts [T, hidden]
    int* err;
};
int flash_forward_tc_q8(const InferAttn& a, cudaStream_t s);
int flash_backward(const fa::Args& a, int max_tiles, int T, cudaStream_t s);

// ---- train_kernels.cu
namespace tr {
struct Mask { float p; float keep; uint64_t seed; };   // inverted dropout by the counter hash; p = 0: identity
struct LnFwd {
    int rows, n;
    const float* x; const int32_t* gather;                  // row r reads x[gather ? gather[r] : r]
    const int32_t* ids; const float* table; int vocab;      // or an embedding gather
    const float* w; const float* b; float eps;
    int identity;                                           // layer 0: y16 = bf16(x)
    __nv_bfloat16* y16; float* y32;                         // outputs (either may be null)
    __nv_bfloat16* y16lo;                                   // with y16: the bf16 remainder y − bf16(y), or null
    float* mean; float* rstd;
    const float* temb; const int32_t* tok_item; const int32_t* qtype;   // y32 += type embedding
    int* err;
};
struct LnBwd {
    int rows, n;
    const float* x; const int32_t* gather;                  // forward input rows
    const float* mean; const float* rstd; const float* w;
    const float* dy;                                        // [rows, n]
    float* dx; int accumulate; const int32_t* scatter;      // dx rows (+= when accumulate, atomic += when scatter)
    float* dw; float* db;                                   // parameter gradients (+=), may be null
    float* part;                                            // scratch for per-CTA dγ/dβ partials ([ctas][2n]), or null
};
constexpr int LN_PART_CTAS_PER_SM = 1;                      // ln_bwd's persistent grid: part holds SMs × this × 2n floats
struct AdamArgs {
    size_t n;
    float* param; const float* grad; float* m; float* v; __nv_bfloat16* shadow; __nv_bfloat16* shadow_lo;
    float decay, b1, b2, step_size, sqrt_c2, eps;
    const double* gscale;                                   // clip factor (device), may be null
};
struct RlcdArgs {
    int n_items, groups, M;                                 // items, noise groups, options (markers)
    const int32_t* mk_start; const int32_t* mk_count; const int32_t* qtype;
    const float* logits; const float* targets; const double* draws;   // draws [groups][M] standard normal
    double sigma, scale, w_sph, w_rps, w_ce;
    double* scratch;                                        // rlcd_scratch_bytes()
    float* dlogits;                                         // [M]
    double* result;                                         // loss, policy loss, cross-entropy, mean reward
};
}  // namespace tr
size_t rlcd_scratch_bytes(int groups, int n_items, int M);
int rlcd(const tr::RlcdArgs& a, cudaStream_t s);
int ln_fwd(const tr::LnFwd& a, cudaStream_t s);
int ln_bwd(const tr::LnBwd& a, cudaStream_t s);
int geglu_fwd(const __nv_bfloat16* wide, int rows, int I, __nv_bfloat16* act, cudaStream_t s);
int geglu_bwd(const __nv_bfloat16* wide, const float* dact, int rows, int I, __nv_bfloat16* dwide, cudaStream_t s);
int geglu_fwd_f32(const float* wide, int rows, int I, __nv_bfloat16* act, __nv_bfloat16* act_lo, cudaStream_t s);
int geglu_bwd_f32(const float* wide, const float* dact, int rows, int I, __nv_bfloat16* dwide, cudaStream_t s);
int relu_mask_f32(const float* pre, __nv_bfloat16* act, __nv_bfloat16* act_lo, size_t n, tr::Mask m, cudaStream_t s);
int relu_mask_bwd_f32(const float* d, const float* pre, __nv_bfloat16* dx, size_t n, tr::Mask m, cudaStream_t s);
int add_masked(const float* a, const float* b, float* y, size_t n, tr::Mask m, cudaStream_t s);
int relu_mask(const __nv_bfloat16* pre, __nv_bfloat16* act, size_t n, tr::Mask m, cudaStream_t s);
int relu_mask_bwd(const float* d, const __nv_bfloat16* pre, __nv_bfloat16* dx, size_t n, tr::Mask m, cudaStream_t s);
int cast_mask(const float* x, __nv_bfloat16* y, size_t n, tr::Mask m, cudaStream_t s);
int f32_to_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s);
int f32_split_bf16(const float* x, __nv_bfloat16* hi, __nv_bfloat16* lo, size_t n, cudaStream_t s);   // lo may be null
int scatter_rows(const float* d, const int32_t* ids, int rows, int n, float* grad, cudaStream_t s);
int colsum_f32(const float* d, int rows, int n, float* db, cudaStream_t s);
int colsum_bf16(const __nv_bfloat16* d, int rows, int n, float* db, cudaStream_t s);
int type_grad(const float* d, const int32_t* tok_item, const int32_t* qtype, int rows, int n, float* grad, cudaStream_t s);
int scorer_out(const float* pre, int M, int n, const float* w2, const float* b2, float* logits, cudaStream_t s);
int scorer_bwd(const float* pre, const float* dlogit, int M, int n, const float* w2, __nv_bfloat16* dpre, float* db1,
               float* dw2, float* db2, cudaStream_t s);
// Σ g² in a fixed order: SUMSQ_BLOCKS per-block partials (no atomics), summed by clip_scale in a fixed tree, so that
// ranks holding the same gradient compute the same norm bit for bit.
constexpr int SUMSQ_BLOCKS = 148 * 8;
int sumsq(const float* g, size_t n, double* partials, cudaStream_t s);
int clip_scale(const double* partials, double max_norm, int world, double* sumsq, double* scale, double* norm_out,
               cudaStream_t s);
int adamw(const tr::AdamArgs& a, cudaStream_t s);

}  // namespace laya
