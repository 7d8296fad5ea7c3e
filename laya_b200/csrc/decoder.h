// decoder.h — argument blocks and launchers of the Mica decoder kernels (decoder_kernels.cu); internal to the library.
//
// Token layout: the rows of all sequences of one forward packed back to back (T rows); seq_start / seq_len give each
// sequence's rows and tok_seq the sequence of every row.  Every activation is row-major [T, width] fp32 unless noted.
// A sequence may continue a state: pos0[s] tokens already read, whose keys and values sit in the state's caches
// (kc / vc [positions, kv·hd] fp16), conv tail (tails [K−1, cd]) and delta-rule state (rec [vh, dk, dv]).  Pointer
// tables are device arrays with one entry per sequence (an entry of 0: no state — zero history, nothing kept).
// Snapshots: snap_begin [n_seq + 1] delimits each sequence's checkpoints snap_at (token counts of its read,
// ascending), and the snapshot states' tails / rec receive the state after that many tokens.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace laya {
namespace dec {

// RMSNorm of rows (row r reads x[row_map ? row_map[r] : r]) · scale (= 1 + weight), optionally kept in fp32 (out32
// [rows, n]) and/or quantized to Q8_0 (q [rows, n], d [n/32, ldd]).
struct RmsArgs {
    int rows, n;
    const float* x;
    const int32_t* row_map;
    const float* scale;
    float eps;
    float* out32;
    q8::code_t* q; float* d; int ldd;
};

// Causal depthwise conv over the first cd columns of in (row stride ld_in), taps w [K, cd] (tap-major), then SiLU.
struct ConvArgs {
    int T, cd, K;
    const float* in; int ld_in;
    const float* w;
    const int32_t* tok_seq; const int32_t* seq_start;
    float* const* tails;   // per sequence (may be null): its history before the first row
    float* out;   // [T, cd]
};

// After the conv: each snapshot's tail and then each state's own tail (the last K−1 pre-conv rows of its history).
struct ConvStateArgs {
    int n_seq, cd, K;
    const float* in; int ld_in;
    const int32_t* seq_start; const int32_t* seq_len;
    float* const* tails;
    const int32_t* snap_begin; const int32_t* snap_at; float* const* snap_tails;
};

// In place on conv [T, cd] = [q (kh·dk) | k (kh·dk) | v]: L2 norm of every q head (· qscale) and k head; β and the
// decay per (row, value head) from the b and a columns of the input projection.
struct HeadsArgs {
    int T, kh, vh, dk, key_dim, cd;
    float* conv;
    float qscale;
    const float* proj; int ld_proj, b_col, a_col;
    const float* dt_bias; const float* neg_a;   // [vh]; neg_a = −exp(A_log)
    float* beta; float* decay;                  // [T, vh]
};

// The gated delta rule, one CTA per (sequence, value head): q, k, v from conv, output [T, ld_out] at h·dv.
struct DeltaArgs {
    int dk, dv, vh, ratio, key_dim, cd;
    const float* conv;
    const float* beta; const float* decay;
    const int32_t* seq_start; const int32_t* seq_len;
    float* out; int ld_out;
    float* const* rec;   // per sequence (may be null): initial state in, final state out
    const int32_t* snap_begin; const int32_t* snap_at; float* const* snap_rec;   // may be null
    int* err;            // device error word (the chunked kernel's bounded waits)
    bool chunked = false;   // a stateless read may take the chunked form (delta_chunk.cu)
};

// RmsNormGated per (row, value head): weight · rmsnorm(core) · silu(z).
struct GatedArgs {
    int T, vh, dv;
    const float* core; int ld_core;
    const float* z; int ld_z;
    const float* weight;
    float eps;
    float* out; int ld_out;
};

// Full attention input: qkv [T, ld_qkv] = [q_h | gate_h for each head h (2·hd each) | k (kv·hd) | v (kv·hd)].
struct PrepArgs {
    int T, heads, kv_heads, hd, half, q_width;
    const float* qkv; int ld_qkv;
    const float* qnorm; const float* knorm;   // 1 + weight
    float eps;
    const float* cosv; const float* sinv;     // [positions, half]
    const int32_t* tok_seq; const int32_t* seq_start; const int32_t* pos0;
    __half* q16;                              // [T, heads·hd]
    __half* const* kc; __half* const* vc;     // per sequence: rows at positions pos0 + (t − seq_start)
};

// Causal GQA attention over 64-query tiles (tile_seq, tile_p0), output · sigmoid(gate) into out [T, ld_out].
struct AttnArgs {
    int heads, kv_heads;
    const __half* q16;
    __half* const* kc; __half* const* vc;   // per sequence: keys and values of positions [0, pos0 + seq_len)
    const int32_t* tile_seq; const int32_t* tile_p0;
    const int32_t* seq_start; const int32_t* seq_len; const int32_t* pos0;
    float scale;
    const float* qkv; int ld_qkv;   // the gates
    float* out; int ld_out;
    int* err = nullptr;   // device error word (the tcgen05 kernel's bounded waits)
};

// Label logits: per (sequence, label) the Q8_0 product of the sequence's final hidden codes with the label's row
// of the Q8_0 token table.
struct LogitArgs {
    int n_seq, n_labels, n, vocab;
    const q8::code_t* qx; const float* dx; int ldx;
    const q8::code_t* qw; const float* dw; int ldw;
    const int32_t* labels;
    float* logits;
    int* err;
};

}  // namespace dec

int dec_rms_q8(const dec::RmsArgs& a, cudaStream_t s);
int dec_embed(const int32_t* ids, int T, int n, int vocab, const q8::code_t* q, const float* d, int ldd, float* x,
              int* err, cudaStream_t s);
int dec_conv_silu(const dec::ConvArgs& a, cudaStream_t s);
int dec_conv_state(const dec::ConvStateArgs& a, cudaStream_t s);
int dec_deltanet_heads(const dec::HeadsArgs& a, cudaStream_t s);
int dec_delta_rule(const dec::DeltaArgs& a, int n_seq, cudaStream_t s);
// delta_chunk.cu: stateless reads at key/value head dims 128 (ERR_NOT_SUPPORTED otherwise)
int dec_delta_rule_chunked(const dec::DeltaArgs& a, int n_seq, cudaStream_t s);
int dec_gated_norm(const dec::GatedArgs& a, cudaStream_t s);
int dec_attn_prep(const dec::PrepArgs& a, cudaStream_t s);
int dec_attention(const dec::AttnArgs& a, int n_tiles, int hd, cudaStream_t s);
// dec_attn_tc.cu: the tcgen05 form for head_dim 128 (ERR_NOT_SUPPORTED for anything else)
int dec_attention_tc(const dec::AttnArgs& a, int n_tiles, int hd, cudaStream_t s);
int dec_add(float* x, const float* y, size_t n, cudaStream_t s);
int dec_gather_rows(const float* src, int ld_src, const int32_t* map, int rows, int n, float* dst, int ld_dst,
                    cudaStream_t s);
int dec_q8_logits(const dec::LogitArgs& a, cudaStream_t s);

}  // namespace laya
