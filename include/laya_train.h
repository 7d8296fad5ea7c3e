/*
 * laya_train.h — C ABI of the fine-tuning step (bf16 tensor-core products, fp32 master weights, AdamW).
 *
 * Replaces the Laya.Training path that Trainer.Train drives (Laya.Training/Trainer.cs:79-154):
 *   TrainableDecisionModel.Forward / Backward      (TrainableDecisionModel.cs:248-353, 479-549)
 *   RlcdObjective.Compute (supplied draws)         (RlcdObjective.cs:57-155)
 *   Gradients.ClipByGlobalNorm, AdamW.Step         (AdamW.cs:29-73, 103-130)
 *   TrainableDecisionModel.ZeroGradients / SetTrainableEncoderLayers  (TrainableDecisionModel.cs:206-238)
 *   Parameter.Data / Gradient                      (Parameter.cs:33-46)
 * and the data-parallel gradient allreduce of the reference notebook's DDP loop (25 MB buckets over NCCL).
 *
 * Conventions are those of laya_b200.h: int status (LAYA_OK = 0), laya_last_error() for the message, host pointers
 * unless a name ends in _device, one trainer per host thread.  Parameter names are the safetensors names
 * TrainableDecisionModel reads (TrainableDecisionModel.cs:111-178).
 *
 * A step, as Trainer.Train runs it:
 *     laya_batch_set(...)                 ids, segments, markers, targets, noise draws -> device
 *     laya_train_forward(t, b, 1, seed)   logits stay on the device (or come back when a buffer is given)
 *     laya_train_objective(t, b, &o, r)   loss + d loss / d logits on the device
 *     laya_train_backward(t, b, NULL)     gradients accumulate (+=) on the device; DP buckets start as they finish
 *     laya_train_clip_and_step(t, ...)    allreduce wait, clip, AdamW, bf16 copies refreshed
 *     laya_train_zero_grads(t)
 */
#ifndef LAYA_TRAIN_H
#define LAYA_TRAIN_H

#include "laya_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct laya_trainer laya_trainer;
typedef struct laya_batch laya_batch;

/* Training options (TrainerOptions, Trainer.cs:16-58; AdamW defaults, AdamW.cs:21-22). */
typedef struct laya_train_desc {
    int trainable_encoder_layers;  /* SetTrainableEncoderLayers: < 0 trains everything incl. embeddings;
                                      n trains the top n encoder layers and the final norm; 0 freezes the encoder */
    float head_dropout;            /* TrainableDecisionModel.HeadDropout (0.1), active when forward's training != 0 */
    double beta1, beta2, eps, weight_decay;  /* 0.9, 0.999, 1e-8, 0.01 */
    double encoder_lr, head_lr;    /* group rates (group 0: names with "encoder.", group 1: the rest) */
    int max_segment;               /* longest segment a batch may carry (rotary tables); <= 2^21 */
    int grad_accumulation;         /* GradientAccumulation: micro-batches per optimizer step (data parallel: the
                                      allreduce overlaps the backward of the last one); <= 0 means 1 */
    int forward_mode;              /* LAYA_FORWARD_ACCURATE (0) or LAYA_FORWARD_BF16 (1), below */
} laya_train_desc;

/* Forward precision of the fine-tuning step.  The backward products are bf16 (fp32 accumulation) in both modes.
 *   ACCURATE  every forward product (projections, attention scores and P·V) is formed from bf16 hi/lo parts of fp32
 *             operands as hi·hi + lo·hi + hi·lo on the tensor cores — fp32-accurate activations, so ReLU masks and
 *             every downstream gradient follow the fp32 reference path (Laya.Training runs fp32).  3x the forward
 *             tensor work.
 *   BF16      forward products from bf16 operands, as torch.autocast(bfloat16) runs the reference notebook's DDP
 *             recipe: fastest, but a bf16 forward moves activations by ~1e-3 relative, which flips ReLU masks of the
 *             decision head and so moves gradients away from the fp32 path by more than rounding. */
#define LAYA_FORWARD_ACCURATE 0
#define LAYA_FORWARD_BF16 1

/* RlcdObjective settings (RlcdObjective.cs:31-35) and the per-call sigma and gradient scale. */
typedef struct laya_rlcd_desc {
    int groups;                    /* GroupSize (4); must match the draws given to laya_batch_set */
    double sigma;                  /* noise scale of this epoch */
    double scale;                  /* 1 / GradientAccumulation */
    double spherical_weight;       /* 0.75 */
    double rps_weight;             /* 1.0 */
    double cross_entropy_weight;   /* 1.0 */
} laya_rlcd_desc;

/* Creates a trainer on `device` for the geometry in `model` (precision is ignored: training is bf16 products over
 * fp32 masters).  Capacity: model->max_tokens tokens, max_items items, max_markers options per batch.
 * Replaces TrainableDecisionModel.FromDirectory + SetTrainableEncoderLayers (TrainableDecisionModel.cs:191-231). */
int laya_trainer_create(const laya_model_desc* model, const laya_train_desc* train, int device, laya_trainer** out);
int laya_trainer_destroy(laya_trainer* t);
/* Stream the trainer enqueues on (NULL: the legacy default stream); by default a stream of its own. */
int laya_trainer_set_stream(laya_trainer* t, void* stream);
int laya_trainer_get_stream(laya_trainer* t, void** stream);
int laya_trainer_synchronize(laya_trainer* t);

/* Parameter data by safetensors name: dtype LAYA_F32, LAYA_BF16 or LAYA_F16 (widened to the fp32 master), shape as
 * stored.  Unknown names or shapes: LAYA_ERR_NOT_FOUND / LAYA_ERR_ARGUMENT.  Parameter.Data (Parameter.cs:33). */
int laya_trainer_upload(laya_trainer* t, const char* name, int dtype, const int64_t* shape, int rank, const void* host);
int laya_trainer_download(laya_trainer* t, const char* name, float* host, int64_t count);
/* The accumulated gradient (Parameter.Gradient, Parameter.cs:40-46); zeros for frozen or untouched parameters. */
int laya_trainer_download_grad(laya_trainer* t, const char* name, float* host, int64_t count);
/* ParameterCount / TrainableParameterCount (TrainableDecisionModel.cs:233-235); temperature excluded. */
int laya_trainer_param_count(laya_trainer* t, int64_t* total, int64_t* trainable);
/* Number of parameter tensors and the i-th one's name (for checkpoint loops). */
int laya_trainer_param_info(laya_trainer* t, int index, const char** name, int64_t* rows, int64_t* cols);
/* Temperature calibration.  laya_temperature_fit: TemperatureFit (TemperatureFitting.cs:10-11) — the per-type
 * temperatures (choice, score, noul; 1.2 for a type without samples) and every "type:size" bucket
 * (QuestionTypes.TemperatureBucket, Base/Questions.cs:38-42) in first-seen order with its sample count, fitted when it
 * has at least min_bucket_samples; every temperature clamped to [0.5, 5] (Calibration.ClampTemperature).
 *   laya_fit_temperatures: TemperatureFitting.Fit (:78-101) on host samples — per sample its question type, option
 *       count, and that many logits and targets, concatenated.  No device work.
 *   laya_train_calibrate: Trainer.Calibrate (Laya.Training/Trainer.cs:200-211) — forward-only passes (no dropout) of
 *       the batches on the device, then the same fit on their option logits and the batches' targets. */
#define LAYA_MAX_TEMPERATURE_BUCKETS 12
typedef struct {
    float by_type[3];
    int n_buckets;
    char bucket[LAYA_MAX_TEMPERATURE_BUCKETS][16];
    int bucket_count[LAYA_MAX_TEMPERATURE_BUCKETS];
    int bucket_fitted[LAYA_MAX_TEMPERATURE_BUCKETS];
    float bucket_temperature[LAYA_MAX_TEMPERATURE_BUCKETS];
} laya_temperature_fit;
int laya_fit_temperatures(const int32_t* qtype, const int32_t* options, const float* logits, const float* targets,
                          int n, int min_bucket_samples, laya_temperature_fit* fit);
int laya_train_calibrate(laya_trainer* t, laya_batch* const* batches, int n_batches, int min_bucket_samples,
                         laya_temperature_fit* fit);

/* Checkpoints.  save: TrainableDecisionModel.Save's model.safetensors (TrainableDecisionModel.cs:649-661,
 * SafetensorsWriter.cs:17-64) — every parameter by name in the dtype it was uploaded in (F32 / F16 / BF16, rounded to
 * nearest even), written to path + ".tmp" then moved over path; with_optimizer != 0 adds AdamW's m and v
 * ("optimizer.m.<name>", "optimizer.v.<name>", F32) and the step count ("__metadata__": "optimizer_step"), which the
 * reference does not save.  restore: reads such a file (or the reference's): every parameter must be present with
 * its shape; the optimizer state and step count come back when present and are reset otherwise. */
int laya_trainer_save_checkpoint(laya_trainer* t, const char* path, int with_optimizer);
int laya_trainer_restore_checkpoint(laya_trainer* t, const char* path);

/* A batch resident on the device: TrainingItem token ids, question types, marker positions and soft targets,
 * plus the standard-normal draws of the objective ([groups][options] in item order, RlcdObjective.cs:57-66).
 * Segments are concatenated without padding as TrainableDecisionModel.Forward does (:253-275).  Token ids outside
 * the vocabulary, or a marker position at or past its segment's end: LAYA_ERR_OUT_OF_RANGE. */
int laya_batch_create(laya_trainer* t, laya_batch** out);
int laya_batch_destroy(laya_batch* b);
int laya_batch_set(laya_trainer* t, laya_batch* b, const int32_t* ids, const int32_t* seg_len, const int32_t* qtype,
                   int n_items, const int32_t* marker_count, const int32_t* markers, const float* targets,
                   const double* draws, int groups);
/* Tokens, items and options the batch holds. */
int laya_batch_shape(laya_batch* b, int* tokens, int* items, int* options);

/* TrainableDecisionModel.Forward(items, training, keepTape: true, seed) (TrainableDecisionModel.cs:248-353): the tape
 * stays on the device for laya_train_backward.  logits: host [options] or NULL (results stay on the device). */
int laya_train_forward(laya_trainer* t, laya_batch* b, int training, uint64_t seed, float* logits);
/* RlcdObjective.Compute(items, logits, sigma, draws, scale) on the logits of the last forward; d loss / d logits stay
 * on the device for laya_train_backward.  result: host [4] = loss, policy loss, cross-entropy, mean reward, or NULL;
 * dlogits: host [options] = ObjectiveResult.LogitGradients in item order, or NULL. */
int laya_train_objective(laya_trainer* t, laya_batch* b, const laya_rlcd_desc* o, double* result, float* dlogits);
/* TrainableDecisionModel.Backward(tape, dlogits) (TrainableDecisionModel.cs:479-549): accumulates (+=) every
 * trainable gradient.  dlogits: host [options], or NULL for the objective's. */
int laya_train_backward(laya_trainer* t, laya_batch* b, const float* dlogits);
/* Group learning rates for the next step (CosineSchedule.Step writes them, AdamW.cs:84-88). */
int laya_train_set_lr(laya_trainer* t, const double* lr, int ngroups);
/* Gradients.ClipByGlobalNorm(max_norm) then AdamW.Step (AdamW.cs:29-73, 103-130) over the trainable parameters.
 * Data-parallel: the gradients are first summed over the ranks (laya_train_comm_init) and averaged.
 * max_norm <= 0: no clipping.  norm: host, the global norm before clipping, or NULL (no synchronisation). */
int laya_train_clip_and_step(laya_trainer* t, double max_norm, double* norm);
/* ZeroGradients (TrainableDecisionModel.cs:237-240). */
int laya_train_zero_grads(laya_trainer* t);
/* AdamW.Steps. */
int laya_train_steps(laya_trainer* t, int64_t* steps);

/* Kernels this host thread has launched through the library (all trainers and contexts). */
int laya_trainer_launches(laya_trainer* t, long long* count);
/* Measurement: with profiling on, every tensor-core product (kind 0), attention forward (1) and attention backward (2)
 * launch is bracketed by CUDA events on the trainer's stream; laya_trainer_profile returns and clears the summed
 * milliseconds, algorithmic FLOPs (2·M·N·K per product whatever its passes; 4·hidden per visible query-key pair
 * forward, twice that backward) and launch count of a kind.  No reference counterpart. */
int laya_trainer_set_profiling(laya_trainer* t, int enabled);
int laya_trainer_profile(laya_trainer* t, int kind, double* ms, double* flops, long long* launches);

/* Data parallelism over NCCL (the reference notebook's DDP; no counterpart in the C# trainer).
 * laya_comm_unique_id fills 128 bytes on one rank; every rank passes the same bytes to laya_train_comm_init.
 * Gradients are then allreduced in 25 MB buckets on a stream of their own as the backward finishes them. */
int laya_comm_unique_id(void* id128);
int laya_train_comm_init(laya_trainer* t, const void* id128, int rank, int world);

#ifdef __cplusplus
}
#endif
#endif /* LAYA_TRAIN_H */
