/*
 * laya_decoder.h — C ABI of the Mica decoder (Qwen3.5 hybrid: Gated DeltaNet ×3 then gated GQA full attention,
 * SwiGLU MLPs, tied Q8_0 token table) on one B200, forward-only prefill scoring with every product in Q8_0.
 *
 * Replaces, for the path the reference runs on its CPU cores:
 *   laya_decoder_create / upload      Qwen35Model(config, weights, WeightPrecision.Q8_0) — the constructor with the
 *                                     Q8_0 stack switch (src/StructuredDecisions.Mica/Models/Qwen35Model.cs:277-337,
 *                                     Stack :361-405, the Q8_0 switch :374-380) and Qwen35Config.FromJson
 *                                     (Qwen35Config.cs:63-135) for the geometry
 *   laya_decoder_forward              Qwen35Model.Forward(IReadOnlyList<Qwen35Sequence>) (Qwen35Model.cs:462-532):
 *                                     every sequence read from an empty state, Readout = true; Hidden = the final
 *                                     RMSNorm of each sequence's last row (:507-518) — followed by
 *                                     Qwen35Model.Logits(hidden, ids, logits) (:586-599 → TokenTable.QuantizedLogits
 *                                     :1091-1111) for the label ids, the call MicaJudge makes (MicaJudge.cs:265-267)
 *   laya_decoder_logits               Qwen35Model.Logits alone, for hidden states the caller holds
 *   laya_decoder_layer                one layer of Forward's loop body (:485-500) on a caller-given hidden state
 *                                     (teacher-forced parity of a single layer; not in the reference's surface)
 *   laya_decoder_record_*             the IStateRecorder of Forward (:468, :505-509, :519-528): "embeddings",
 *                                     "layers.{i}.mixer", "layers.{i}", "norm"
 *   laya_decoder_state_* / _mark_*    Qwen35State (:38-197): NewState, Clone, Save / Rewind, Length, Bytes, Dispose
 *   laya_decoder_forward_states       Forward over sequences that continue states, with in-pass Checkpoints
 *                                     (:462-532, :734-749, :880-895) — Mica's shared-prefix reuse (MicaJudge.cs:166-229)
 *
 * Weights are the Hugging Face checkpoint's tensors by name ("model." or "model.language_model." prefixes are
 * accepted and dropped).  Projections (q/k/v/o, in_proj_*, out_proj, gate/up/down) and embed_tokens are kept as Q8_0:
 * uploaded as fp32/bf16 they are quantized on the device exactly as the reference quantizes them at load
 * (PackedMatrixQ8_0.QuantizeWeightBlock); uploaded pre-quantized (laya_decoder_upload_q8_0) they are taken as given.
 * Sibling projections are stacked along the output, one product each (in_proj_qkv|z|b|a; q|k|v; gate|up), as the
 * reference's Stack does.  Norm weights are stored as 1 + w (the zero-centred RMSNorm), except the DeltaNet's gated
 * norm, which uses w itself.  A_log is stored as −exp(A_log).
 *
 * Status codes, dtypes and laya_last_error() are those of laya_b200.h.  Thread safety: one decoder per host thread
 * at a time; calls are asynchronous on the decoder's stream except those that return host data.
 */
#ifndef LAYA_DECODER_H
#define LAYA_DECODER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct laya_decoder laya_decoder;

/* Layer kinds of laya_decoder_desc.layer_kinds (Qwen35Config.LayerTypes: "linear_attention" / "full_attention"). */
#define LAYA_DECODER_LINEAR 0
#define LAYA_DECODER_FULL 1

/* Qwen35Config (Qwen35Config.cs:60-130) plus the capacity of one forward. */
typedef struct {
    int hidden;             /* hidden_size; a multiple of 32 */
    int intermediate;       /* intermediate_size; a multiple of 32 */
    int layers;             /* num_hidden_layers */
    int vocab;              /* vocab_size */
    float eps;              /* rms_norm_eps */
    const int32_t* layer_kinds;   /* [layers], LAYA_DECODER_LINEAR / LAYA_DECODER_FULL (copied at create) */
    int heads;              /* num_attention_heads */
    int kv_heads;           /* num_key_value_heads; divides heads */
    int head_dim;           /* 32, 64 or 128 */
    double rope_theta;      /* rope_parameters.rope_theta */
    int rotary_dim;         /* head_dim · partial_rotary_factor; even, ≤ head_dim */
    int lin_k_heads;        /* linear_num_key_heads */
    int lin_v_heads;        /* linear_num_value_heads; a multiple of lin_k_heads */
    int lin_k_dim;          /* linear_key_head_dim: 16, 32, 64 or 128 */
    int lin_v_dim;          /* linear_value_head_dim: ≤ 128 */
    int conv_kernel;        /* linear_conv_kernel_dim */
    int max_tokens;         /* rows of one forward (all sequences together) */
    int max_seqs;           /* sequences of one forward */
} laya_decoder_desc;

int laya_decoder_create(const laya_decoder_desc* desc, int device, laya_decoder** out);
int laya_decoder_destroy(laya_decoder* dec);
int laya_decoder_set_stream(laya_decoder* dec, void* stream);   /* a cudaStream_t; NULL = the decoder's own */
int laya_decoder_get_stream(laya_decoder* dec, void** stream);
int laya_decoder_synchronize(laya_decoder* dec);

/* One checkpoint tensor by name; dtype LAYA_F32 / LAYA_BF16 / LAYA_F16. */
int laya_decoder_upload(laya_decoder* dec, const char* name, int dtype, const int64_t* shape, int rank,
                        const void* host);
/* A projection or embed_tokens already in Q8_0: q [N, K] int8 codes, d_fp16 [N, K/32] block scales (fp16 bits). */
int laya_decoder_upload_q8_0(laya_decoder* dec, const char* name, const int8_t* q, const uint16_t* d_fp16, int N,
                             int K);
/* Names still missing before a forward can run: writes up to `cap` bytes of a newline-separated list into `names`
 * (may be NULL) and the count into *missing. */
int laya_decoder_missing(laya_decoder* dec, char* names, int cap, int* missing);

/* Prefill scoring of n_seq sequences (ids packed back to back, seq_len[s] rows each, every length ≥ 1), each from an
 * empty state.  hidden [n_seq, hidden] (may be NULL): each sequence's final-normed last row; logits
 * [n_seq, n_labels] (may be NULL): the tied head's logits of label_ids at that row.  Host buffers; returns when the
 * results are on the host.  Token or label ids outside the vocabulary: LAYA_ERR_OUT_OF_RANGE. */
int laya_decoder_forward(laya_decoder* dec, const int32_t* ids, const int32_t* seq_len, int n_seq,
                         const int32_t* label_ids, int n_labels, float* hidden, float* logits);
/* The same with ids, hidden and logits in device memory (seq_len and label_ids stay host arrays); asynchronous on
 * the decoder's stream (id errors surface at the next synchronizing call). */
int laya_decoder_forward_device(laya_decoder* dec, const int32_t* ids, const int32_t* seq_len, int n_seq,
                                const int32_t* label_ids, int n_labels, float* hidden, float* logits);
/* Qwen35Model.Logits: rows of hidden [rows, hidden] (host) against the token table's rows `ids` → logits
 * [rows, n_ids]. */
int laya_decoder_logits(laya_decoder* dec, const float* hidden, int rows, const int32_t* ids, int n_ids,
                        float* logits);
/* One decoder layer on hidden [T, hidden] (host, in place), T = Σ seq_len; mixer (may be NULL) receives the
 * layer's mixer output (before its residual add). */
int laya_decoder_layer(laya_decoder* dec, int layer, float* hidden, const int32_t* seq_len, int n_seq,
                       float* mixer);

/* States (Qwen35State, Qwen35Model.cs:38-197): what the decoder remembers of the tokens a sequence has read, in device
 * memory — keys and values of every full-attention layer (fp16 [capacity, kv_heads·head_dim], normed and rotated as
 * attention reads them), and the conv tail [conv_kernel − 1, conv dim] plus the delta-rule state
 * [lin_v_heads, lin_k_dim, lin_v_dim] (fp32) of every DeltaNet layer.  Reading a prompt in several forwards through
 * one state gives bit for bit the hidden state and logits of reading it in one forward.  State calls are
 * asynchronous on the decoder's stream; a state belongs to the decoder that made it (destroying the decoder frees
 * its states' memory; the handles must still be destroyed). */
typedef struct laya_decoder_state laya_decoder_state;
typedef struct laya_decoder_mark laya_decoder_mark;

/* Qwen35Model.NewState (:419): a state that has read nothing, with room for `capacity` tokens (a hint: the key and
 * value caches grow on demand to the next power of two, as Qwen35State.GrowCache does, :146-154). */
int laya_decoder_state_create(laya_decoder* dec, int capacity, laya_decoder_state** out);
/* Qwen35State.Dispose (:187-196). */
int laya_decoder_state_destroy(laya_decoder_state* state);
/* Qwen35State.Length (:62) and Bytes (:183-184): tokens read; device bytes held. */
int laya_decoder_state_length(const laya_decoder_state* state, int* length);
int laya_decoder_state_bytes(const laya_decoder_state* state, int64_t* bytes);
/* Qwen35State.Clone (:112-117): an independent copy — what is read into one never reaches the other. */
int laya_decoder_state_clone(laya_decoder_state* state, laya_decoder_state** out);
/* Qwen35State.Save (:127-131) / Rewind (:134-143) / Mark.Dispose (:174-180): a mark keeps the length and a copy of the
 * conv tails and delta-rule states; rewinding copies them back and moves the length back (keys and values are not
 * copied: what is read next overwrites them).  A mark longer than the state, or of another decoder:
 * LAYA_ERR_ARGUMENT. */
int laya_decoder_state_save(laya_decoder_state* state, laya_decoder_mark** out);
int laya_decoder_state_rewind(laya_decoder_state* state, const laya_decoder_mark* mark);
int laya_decoder_mark_destroy(laya_decoder_mark* mark);

/* Qwen35Model.Forward(IReadOnlyList<Qwen35Sequence>) (:462-532) over states: sequence s reads its seq_len[s] tokens
 * after what states[s] holds and advances it (n_seq distinct states of this decoder).  readout [n_seq] (may be
 * NULL) is Qwen35Sequence.Readout; hidden / logits rows are written for every sequence and meaningful for those
 * with readout.  Checkpoints (Qwen35Sequence.Checkpoints / Snapshots, :214-221; MicaJudge.cs:87, :189-212):
 * n_checkpoints [n_seq] (may be NULL), checkpoints the concatenated token counts of each sequence (strictly
 * ascending within 1..seq_len[s]), and snapshots [Σ n_checkpoints] receives one new state per checkpoint — owned by
 * the caller — holding what its sequence held after that many tokens.  Qwen35Model.Read (:437-439) is this call with
 * hidden and logits NULL.  ids, seq_len, label ids and results are host arrays; the call returns when the results are
 * on the host.  Invalid arguments and ids outside the vocabulary are rejected before any state changes. */
int laya_decoder_forward_states(laya_decoder* dec, const int32_t* ids, const int32_t* seq_len, int n_seq,
                                laya_decoder_state* const* states, const int32_t* readout,
                                const int32_t* n_checkpoints, const int32_t* checkpoints,
                                laya_decoder_state** snapshots, const int32_t* label_ids, int n_labels, float* hidden,
                                float* logits);

/* How the DeltaNet layers' delta rule runs for reads without a decoder state (laya_decoder_forward,
 * laya_decoder_layer): 0 (the default) the per-token sweep, bit-identical to DecoderKernels.GatedDeltaRule128
 * (DecoderKernels.cs:151-259), so a stateless read gives the same bits as a read through a state; 1 in 64-token
 * chunks on the tensor cores where the key and value head dims are 128 — fp32-accurate products, so it agrees with
 * the sweep to rounding (~1e-5 relative), not bit for bit, and the Q8_0 activation codes downstream may differ.
 * Reads through states always run the per-token sweep: reading in pieces must give the bits of reading at once
 * (Qwen35State, Qwen35Model.cs:38-197). */
int laya_decoder_set_chunked_delta_rule(laya_decoder* dec, int enabled);

/* Recorder of the next forwards (single or several sequences; rows packed): 1 on, 0 off. */
int laya_decoder_record_enable(laya_decoder* dec, int enabled);
int laya_decoder_record_get(laya_decoder* dec, const char* name, float* host, int64_t count);

/* Kernel launches issued by this host thread so far; profiling of the products (kind 0), the delta rule
 * (kind 1) and full attention (kind 2) by CUDA events: total ms, algorithmic operations, launches. */
int laya_decoder_launches(laya_decoder* dec, long long* count);
int laya_decoder_set_profiling(laya_decoder* dec, int enabled);
int laya_decoder_profile(laya_decoder* dec, int kind, double* ms, double* ops, long long* n);

#ifdef __cplusplus
}
#endif
#endif /* LAYA_DECODER_H */
