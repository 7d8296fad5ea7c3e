/*
 * laya_b200.h — C ABI of the B200 (sm_100a) library behind the Laya decision engine's hot path.
 *
 * Plain C: pointers, sizes and status codes only.  Every function returns an int status (0 = LAYA_OK);
 * laya_last_error() returns the calling thread's message for the last failure.  The host wrapper maps codes
 * to the exceptions the reference throws today (LAYA_ERR_ARGUMENT -> ArgumentException,
 * LAYA_ERR_OUT_OF_RANGE -> ArgumentOutOfRangeException, LAYA_ERR_NOT_SUPPORTED -> PlatformNotSupportedException).
 *
 * Memory: functions named *_device take device pointers and enqueue on the context's stream without
 * synchronising; every other data pointer is host memory, and the call returns after the result is in it.
 * A context owns its device memory (weights, workspaces); the caller owns everything it passes.
 *
 * Threading: one context per host thread; calls on one context are serialised by the caller.
 *
 * Reference interfaces each entry point replaces are cited as file:line inside the reference project
 * (theolivenbaum/laya).
 */
#ifndef LAYA_B200_H
#define LAYA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LAYA_OK 0
#define LAYA_ERR_ARGUMENT 1
#define LAYA_ERR_OUT_OF_RANGE 2
#define LAYA_ERR_NOT_SUPPORTED 3
#define LAYA_ERR_CUDA 4
#define LAYA_ERR_NOT_FOUND 5
#define LAYA_ERR_DEVICE_TIMEOUT 6
#define LAYA_ERR_COMM 7

/* dtypes of laya_upload_tensor */
#define LAYA_F32 0
#define LAYA_BF16 1
#define LAYA_F16 2
#define LAYA_I8 3
#define LAYA_I32 4

/* precision of a model's projections */
#define LAYA_PRECISION_F32 0   /* the reference's PackedMatrix fp32 product */
#define LAYA_PRECISION_Q8_0 1  /* ggml Q8_0 weights and activations (WeightPrecision.Q8_0, PackedMatrixQ8_0.cs:75-81) */

typedef struct laya_ctx laya_ctx;

/*
 * Geometry of the ModernBERT encoder + decision head (ModernBertConfig.FromJson, Laya/Models/ModernBertConfig.cs:60-117;
 * LayaConfig, ModernBertConfig.cs:124-184).  layer_kinds[i] is 1 for a global-attention layer, 0 for a sliding one;
 * NULL means "global every global_every layers, starting at 0".
 */
typedef struct laya_model_desc {
    int hidden;            /* 768 base, 1024 large */
    int intermediate;      /* GeGLU width I (Wi emits 2I) */
    int layers;
    int heads;             /* head_dim = hidden / heads (64) */
    int vocab;
    int local_attention;   /* sliding window; a token sees [i - local_attention/2, i + local_attention/2] */
    int global_every;
    const int* layer_kinds;
    double theta_global;
    double theta_local;
    float norm_eps;        /* encoder LayerNorm eps (bias-free) */
    int head_layers;       /* decision-head transformer layers (2) */
    int n_act;             /* act-head outputs */
    int act_hidden;        /* act-head hidden width (256) */
    int precision;         /* LAYA_PRECISION_* */
    int max_tokens;        /* workspace size: most tokens one forward may carry */
    int max_items;         /* most questions one forward may carry */
    int max_markers;       /* most option markers in one forward */
} laya_model_desc;

/* The calling thread's message for the last failed call ("" if none). */
const char* laya_last_error(void);

/* Version string of the library build. */
const char* laya_version(void);

/* Creates a context on CUDA device `device` for the given geometry.  Replaces the DecisionModel /
 * ModernBertEncoder constructors (Laya/Models/DecisionModel.cs:50-99, ModernBertEncoder.cs:62-102): weights
 * then arrive by name through laya_upload_tensor / laya_upload_q8_0. */
int laya_ctx_create(const laya_model_desc* desc, int device, laya_ctx** out);
int laya_ctx_destroy(laya_ctx* ctx);

/* Makes every later launch of this context go to `stream` (a cudaStream_t); NULL selects CUDA's legacy default
 * stream.  A new context launches on a non-blocking stream of its own; laya_ctx_get_stream returns the current one. */
int laya_ctx_set_stream(laya_ctx* ctx, void* stream);
int laya_ctx_get_stream(laya_ctx* ctx, void** stream);

/* Blocks until the context's stream is idle, then reports any device-side error (a timed-out wait inside
 * a kernel returns LAYA_ERR_DEVICE_TIMEOUT). */
int laya_ctx_synchronize(laya_ctx* ctx);

/* Kernel launches this context issued so far (every laya_b200 kernel counts one). */
int laya_ctx_launches(laya_ctx* ctx, long long* count);

/* Per-launch timing of the Q8_0 products: when enabled, each product launch is bracketed by CUDA events on
 * the context's stream; laya_ctx_profile returns the summed device milliseconds, the summed int8 operations
 * (2·M·N·K) and the number of timed launches since the last reset. */
int laya_ctx_set_profiling(laya_ctx* ctx, int enabled);
int laya_ctx_profile(laya_ctx* ctx, double* gemm_ms, double* gemm_ops, long long* gemm_launches);

/*
 * Uploads one named tensor (safetensors name, as TrainableDecisionModel / DecisionModel read them:
 * TrainableDecisionModel.cs:111-178, DecisionModel.cs:55-91).  dtype LAYA_F32/LAYA_BF16/LAYA_F16 are widened to fp32
 * on the device (SafetensorsFile.ReadFloat32, Base/Io/SafetensorsFile.cs:101-205).  For a Q8_0 context, a projection
 * uploaded as floats is quantized on the device with ggml's weight quantizer (the PackedMatrixQ8_0 constructors,
 * PackedMatrixQ8_0.cs:146-173).
 */
int laya_upload_tensor(laya_ctx* ctx, const char* name, int dtype, const int64_t* shape, int rank, const void* host);

/* Uploads a projection already in Q8_0: codes q [N, K] (int8) and per-32-block scales d_fp16 [N, K/32] (IEEE fp16
 * bits), as a GGUF file stores them (Q8_0 block layout, PackedMatrixQ8_0.cs:101-106). */
int laya_upload_q8_0(laya_ctx* ctx, const char* name, const int8_t* q, const uint16_t* d_fp16, int N, int K);

/* Downloads a tensor uploaded under `name` as fp32 (Q8_0 projections come back dequantized, q·d, as
 * PackedMatrixQ8_0.Dequantize, PackedMatrixQ8_0.cs:209-218). */
int laya_download_tensor(laya_ctx* ctx, const char* name, float* host, int64_t count);

/*
 * ILinear.Multiply for a Q8_0 projection (PackedMatrixQ8_0.Multiply, PackedMatrixQ8_0.cs:220-246; the ILinear
 * interface, Base/Numerics/PackedMatrixBf16.cs:419-430): y[r, 0..N) = Q8_0(x[r, 0..K)) · W + bias, row strides in
 * floats.  `weight` names a projection uploaded to this context; bias may be NULL.  Errors as the reference: short or
 * inconsistent sizes -> LAYA_ERR_ARGUMENT.
 */
int laya_q8_0_linear(laya_ctx* ctx, const char* weight, const float* x, int rows, int input_stride, const float* bias,
                     float* y, int output_stride);
int laya_q8_0_linear_device(laya_ctx* ctx, const char* weight, const float* x, int rows, int input_stride,
                            const float* bias, float* y, int output_stride);

/*
 * The Q8_0 primitives on caller-owned device buffers, in the layouts the kernels use.  On the device a Q8_0 code is
 * held as an IEEE fp16 value equal to the integer code (-127..127; the reference stores q+128 as bytes): the
 * tensor-core product multiplies these exactly.  Block scales are fp32 holding the stored fp16 value.
 *   laya_q8_0_quantize_activations_device: Q8_0.QuantizeActivations (PackedMatrixQ8_0.cs:35-71); x [rows, stride] ->
 *       q [rows, K] codes, d [K/32, ldd] block scales as stored (fp16-rounded).
 *   laya_q8_0_quantize_weights_device: Q8_0.QuantizeWeightBlock over every block (PackedMatrixQ8_0.cs:20-28);
 *       w [N, K] -> q [N, K], d [K/32, ldd].
 *   laya_q8_0_gemm_device: the product of already-quantized operands (the kernels of PackedMatrixQ8_0.cs:248-557);
 *       out[M, N] (row stride ldo) = bias + Σ_b fma(Σ_b, dw·dx); ldx >= M rounded up to 128, ldw >= N, both multiples
 *       of 4; every buffer 16-byte aligned.  Output rows are written in whole 16-byte chunks, so columns
 *       N..roundup(N, 4)-1 of each row (inside the row stride) may be overwritten.
 */
/* The PackedMatrixQ8_0 constructors (PackedMatrixQ8_0.cs:146-173): a PyTorch [N, K] weight given as fp32 (LAYA_F32),
 * bf16 bits (LAYA_BF16) or fp16 bits (LAYA_F16), quantized on the device with ggml's weight quantizer and kept under
 * `name` for laya_q8_0_linear.  K not a multiple of 32 -> LAYA_ERR_ARGUMENT, as the reference throws. */
int laya_pack_q8_0(laya_ctx* ctx, const char* name, int dtype, const void* host, int N, int K);

int laya_q8_0_quantize_activations_device(laya_ctx* ctx, const float* x, int rows, int stride, int K, uint16_t* q,
                                          float* d, int ldd);
int laya_q8_0_quantize_weights_device(laya_ctx* ctx, const float* w, int N, int K, uint16_t* q, float* d, int ldd);
int laya_q8_0_gemm_device(laya_ctx* ctx, const uint16_t* qx, const float* dx, int ldx, int M, const uint16_t* qw,
                          const float* dw, int ldw, int N, int K, const float* bias, float* out, int ldo);

/*
 * The product with one of the fused epilogues the forward uses (each stands for the reference operations that follow
 * a projection, which read the product's fp32 output):
 *   0  out = product                                       (ILinear.Multiply)
 *   1  out += product, in place                           (the residual adds, SimdOps.Add, ModernBertEncoder.cs:174,181)
 *   2  weight rows in GeGLU order — groups of 64 = 32 rows of Wi's first half then the matching 32 of its second half —
 *      and qout/qscale = Q8_0(gelu(u) · g) of the N/2 activations  (ModernBertEncoder.GeGlu, ModernBertEncoder.cs:204-214,
 *      then the next projection's activation quantizer)
 *   3  qout/qscale = Q8_0(relu(product))                  (DecisionModel.cs:300-304)
 *   4  weight rows in SwiGLU order — groups of 64 = 32 gate rows then the matching 32 up rows — and
 *      qout/qscale = Q8_0(silu(g) · u) of the N/2 activations  (Qwen35Model.Mlp, Qwen35Model.cs:602-621, then the
 *      down projection's activation quantizer)
 * qout is [M, N or N/2] codes, qscale [columns/32, ldqs] block scales.
 */
int laya_q8_0_gemm_fused_device(laya_ctx* ctx, int epilogue, const uint16_t* qx, const float* dx, int ldx, int M,
                                const uint16_t* qw, const float* dw, int ldw, int N, int K, const float* bias, float* out,
                                int ldo, uint16_t* qout, float* qscale, int ldqs);

/*
 * The bf16 tensor-core product of the training step on caller device buffers (PackedMatrix.Multiply as Ops.Linear and
 * Ops.LinearBackward use it, Laya.Training/Ops.cs:22-69): out[M, N] = A · Bᵀ (+ bias) with fp32 accumulation.
 * A is [M, K] (a_mn = 0, row stride lda) or stored transposed as [K, lda] (a_mn = 1); likewise B [N, K] or [K, ldb].
 * epilogue 0: out bf16 [M, ldo]; 1: out fp32; 2: out fp32 += product (accumulating gradients and residual streams;
 * when few output tiles cover a long K, K is split into chunks that reduce-add, so the summation order may vary).
 * Bases 16-byte aligned, row strides multiples of 8 elements (4 for fp32 outputs).
 */
int laya_gemm_bf16_device(laya_ctx* ctx, int M, int N, int K, const uint16_t* A, int lda, int a_mn, const uint16_t* B,
                          int ldb, int b_mn, const float* bias, int epilogue, void* out, int ldo);
/*
 * The same product with fp32 accuracy from bf16 tensor cores (the fine-tuning forward's products): the caller passes
 * each fp32 operand as hi = bf16(x) and lo = bf16(x - hi) (same layouts), and gets A·Bᵀ + A_lo·Bᵀ + A·B_loᵀ; with
 * B_lo NULL (B exactly bf16, as a bf16 checkpoint's weights are) A·Bᵀ + A_lo·Bᵀ, two passes instead of three.
 * No reference counterpart beyond PackedMatrix.Multiply's fp32 result, which it reproduces to about 2^-16 relative.
 */
int laya_gemm_bf16_split_device(laya_ctx* ctx, int M, int N, int K, const uint16_t* A, const uint16_t* A_lo, int lda,
                                int a_mn, const uint16_t* B, const uint16_t* B_lo, int ldb, int b_mn, const float* bias,
                                int epilogue, void* out, int ldo);

/*
 * laya_q8_0_linear_noalloc — the Q8_0 projection y = Q8_0(x) · W (+ bias) without any device allocation.
 * No counterpart in the reference: it exists for callers that cannot call cudaMalloc — hosts whose device memory
 * is owned by their own pool under a fixed budget, and plugins inside another process that may neither grow its
 * device footprint nor take the implicit device synchronisation of cudaMalloc/cudaFree on a latency-critical path.
 *   x [rows, input_stride] fp32 and y [rows, output_stride] fp32 are device buffers of the caller (y 16-byte aligned,
 *   output_stride a multiple of 4); weight_codes
 *   [N, K] and weight_scales [K/32, ldw] are a projection in the device layout of laya_q8_0_quantize_weights_device
 *   (16-byte aligned, ldw >= N and a multiple of 4); bias [N] or NULL.  Enqueued on `stream` (NULL: the legacy default
 *   stream).  The call then waits for that stream and reads back the product's status word: a bounded device-side
 *   wait that gave up returns LAYA_ERR_DEVICE_TIMEOUT (message in laya_last_error()), and y is then not valid.
 * The scratch (activation codes, their scales, a status word) is one static device array of LAYA_NOALLOC_SCRATCH_BYTES
 * that every GPU loading the library holds until the process exits; a call needs about rows·K·2 + rows·K/8 bytes of it,
 * and larger calls fail with LAYA_ERR_ARGUMENT before anything runs.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that first call before any stream capture.
 * Every call shares the array: calls that overlap on the GPU (different streams, devices excepted) race and must be
 * serialised by the caller.
 */
#define LAYA_NOALLOC_SCRATCH_BYTES (8u << 20)
int laya_q8_0_linear_noalloc(const float* x, int rows, int input_stride, const uint16_t* weight_codes,
                             const float* weight_scales, int ldw, int N, int K, const float* bias, float* y,
                             int output_stride, void* stream);

/*
 * The batched decision forward (DecisionModel.Forward, Laya/Models/DecisionModel.cs:128-169, with ModernBertEncoder.Forward,
 * ModernBertEncoder.cs:123-188): questions concatenated, not padded.
 *   ids [Σ seg_len]          token ids of every question back to back
 *   seg_len [n_items]        tokens per question
 *   qtype [n_items]          question type (0 choice, 1 score, 2 noul)
 *   marker_count [n_items]   option markers per question
 *   markers [Σ marker_count] marker positions inside each question (negative positions read position 0)
 *   logits [Σ marker_count]  option logits out
 *   act_probs [n_items · n_act] action probabilities out (may be NULL)
 * Token ids outside the vocabulary -> LAYA_ERR_OUT_OF_RANGE (ModernBertEncoder.cs:136-139).
 */
int laya_decision_forward(laya_ctx* ctx, const int32_t* ids, const int32_t* seg_len, const int32_t* qtype, int n_items,
                          const int32_t* marker_count, const int32_t* markers, float* logits, float* act_probs);
/* The same on device buffers, enqueued on the context's stream without synchronising; the caller passes the token and
 * marker totals (Σ seg_len, Σ marker_count).  Check laya_ctx_synchronize for device-side range errors. */
int laya_decision_forward_device(laya_ctx* ctx, const int32_t* ids, const int32_t* seg_len, const int32_t* qtype,
                                 int n_items, int n_tokens, const int32_t* marker_count, const int32_t* markers,
                                 int n_markers, float* logits, float* act_probs);

/* Encoder alone (ModernBertEncoder.Forward, ModernBertEncoder.cs:123-188): final hidden states [Σ seg_len, hidden]. */
int laya_encoder_forward(laya_ctx* ctx, const int32_t* ids, const int32_t* seg_len, int n_items, float* hidden);

/*
 * Recorder hook (IStateRecorder.Record, Base/Diagnostics/StateRecorder.cs:7-9): while enabled, the forward keeps a
 * device copy of the residual stream after every encoder layer and head layer; laya_record_get copies the one named
 * "encoder.layers.{i}.output", "encoder.last_hidden_state" or "head.layers.{i}.output" ([T, hidden] fp32) to host.
 */
int laya_record_enable(laya_ctx* ctx, int enabled);
int laya_record_get(laya_ctx* ctx, const char* name, float* host, int64_t count);

/*
 * One encoder layer on caller-supplied hidden states (teacher forcing for per-layer parity): h [T, hidden] in/out,
 * segments as in laya_encoder_forward.  Runs layer `layer` exactly as the full forward does.
 */
int laya_encoder_layer(laya_ctx* ctx, int layer, float* hidden, const int32_t* seg_len, int n_items);

/*
 * laya_mma_peak — a measurement, not part of the reference's interface (it has no counterpart there): the rate of
 * the tensor cores on the current device for one MMA form, the denominator the library's product kernels are
 * reported against.  One CTA per SM issues `reps` rounds of four back-to-back M 128 × N (64, 128 or 256) MMAs of
 * one 128-byte k-block from fixed shared-memory operands into one TMEM accumulator.  *ms: the launch's elapsed time;
 * *cycles_per_mma: mean SM cycles per MMA instruction seen by the issuing threads.  Work per launch:
 * SMs × reps × 4 × 2 × 128 × N × K (K 16 for the 16-bit forms, 32 for int8).
 */
#define LAYA_MMA_BF16 0      /* kind::f16, bf16 operands, fp32 accumulate */
#define LAYA_MMA_F16 1       /* kind::f16, fp16 operands (the Q8_0 product's form) */
#define LAYA_MMA_I8 2        /* kind::i8, s8 operands, s32 accumulate */
#define LAYA_MMA_BF16_TS 3   /* kind::f16 bf16 with A read from tensor memory */
#define LAYA_MMA_BF16_MN 4   /* kind::f16 bf16 with B read N-contiguous (MN-major) */
#define LAYA_MMA_BF16_TS_MN 5   /* A from tensor memory, B N-contiguous (the attention P·V form) */
int laya_mma_peak(int form, int n, int reps, double* ms, double* cycles_per_mma);

#ifdef __cplusplus
}
#endif

#endif /* LAYA_B200_H */
