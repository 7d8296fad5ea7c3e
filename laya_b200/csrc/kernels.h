// kernels.h — argument blocks and launchers of the laya_b200 kernels (internal to the library).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace laya {

// ---- norm.cu
struct LnArgs {
    int rows, n;
    const float* x;            // [rows, n] input (unused by the embedding gather)
    const int32_t* ids;        // embedding gather: token ids
    const float* table;        // embedding gather: [vocab, n]
    int vocab;
    const float* w;            // LayerNorm weight [n]
    const float* b;            // LayerNorm bias [n] or null
    float eps;
    int apply_ln;              // 0: identity (ModernBERT layer 0 has no attn_norm)
    float* out;                // fp32 output [rows, n]
    const float* temb;         // final LN: type embedding [3, n]
    const int32_t* tok_item;   // final LN: question of each token
    const int32_t* qtype;      // final LN: type of each question
    __half* q; float* d; int ldd;   // Q8_0 output: fp16-held codes [rows, n], scales [n/32, ldd]
    __nv_bfloat16* hi; __nv_bfloat16* lo;   // or (q null) the output split as hi = bf16(y), lo = bf16(y − hi) [rows, n]
    int* err;
};
int ln_q8(const LnArgs& a, cudaStream_t s);
int ln_final(const LnArgs& a, cudaStream_t s);
int ln_embed(const LnArgs& a, cudaStream_t s);

// ---- attention.cu
namespace attn {
struct Args {
    const float* qkv; int ld; int hidden; int heads;
    const int32_t* seg_start; const int32_t* seg_len;
    const int32_t* qtile_item; const int32_t* qtile_q0; const int32_t* n_qtiles;
    int window;                       // < 0: global
    float scale;                      // 1/sqrt(head_dim), applied to every dot product
    const float* cosv; const float* sinv;   // [positions, head_dim/2] or null (no rotary)
    __half* q; float* d; int ldd;     // context codes (fp16-held) [T, hidden], scales [hidden/32, ldd]
    __nv_bfloat16* hi; __nv_bfloat16* lo;   // or (q null) the context split as hi = bf16(c), lo = bf16(c − hi)
};
}  // namespace attn
int attention(const attn::Args& a, int max_qtiles, cudaStream_t stream);

// ---- head.cu
struct PlanArgs {
    int n_items, n_tokens, n_markers, max_qtiles;
    const int32_t* seg_len; const int32_t* marker_count; const int32_t* markers;
    int32_t* seg_start; int32_t* mk_start; int32_t* qt_start;
    int32_t* qt_item; int32_t* qt_q0; int32_t* n_qtiles;
    int32_t* tok_item; int32_t* marker_row; int32_t* marker_item;
    int* err;
    // 128-row query tiles (the tensor-core attention), when tq_start is given
    int max_tq; int32_t* tq_start; int32_t* tq_item; int32_t* tq_p0; int32_t* n_tq;
};
int plan(const PlanArgs& a, cudaStream_t stream);
// fp32 q | k | v rows [T, ld] → fp16 [T, ldo], q and k rotated at the token's position in its segment (cos/sin
// [positions, head_dim/2], or none): the tensor-core attention's operands.
int attn_prep16(const float* qkv, int ld, int T, int hidden, int heads, const int32_t* tok_item, const int32_t* seg_start,
                const float* cosv, const float* sinv, __half* out, int ldo, cudaStream_t stream);

struct ScorerArgs {
    int n_markers, hidden;
    const float* h; const int32_t* marker_row;
    const float* ln_w; const float* ln_b;
    const float* w1; const float* b1; const float* w2; const float* b2;
    float* hid;        // [n_markers, hidden] workspace: GELU(Linear1) of each marker row
    float* logits;
};
int scorer(const ScorerArgs& a, cudaStream_t stream);

struct ActArgs {
    int n_items, hidden, act_hidden, n_act, max_k;
    const float* h; const int32_t* seg_start; const int32_t* mk_start; const int32_t* marker_count;
    const float* logits;
    const float* w1; const float* b1; const float* w2; const float* b2;
    float* probs;
};
int act_head(const ActArgs& a, cudaStream_t stream);

}  // namespace laya
