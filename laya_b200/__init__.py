"""laya_b200 — the Laya decision engine's hot path on B200 (sm_100a), behind a C ABI.

The compute lives in `liblaya_b200.so` (CUDA kernels + the C ABI of include/laya_b200.h).  This package is the
host-side mirror of the reference's interfaces for that path, over ctypes:

  * `DecisionModel`      — DecisionModel / ModernBertEncoder inference (Laya/Models/DecisionModel.cs,
                           Laya/Models/ModernBertEncoder.cs): construct from named weights, `forward(items)`.
  * `PackedMatrixQ8_0`   — the ILinear Q8_0 projection (Base/Numerics/PackedMatrixQ8_0.cs): `multiply(...)`.
  * `Q8_0`               — the quantizers on device buffers.
  * `Trainer`, `Batch`   — the fine-tuning step of include/laya_train.h (Laya.Training/TrainableDecisionModel.cs,
                           RlcdObjective.cs, AdamW.cs): forward, objective, backward, clip + AdamW, NCCL buckets.
  * `Qwen35Model`        — the Mica decoder of include/laya_decoder.h (Mica/Models/Qwen35Model.cs) with Q8_0
                           products: prefill of packed sequences, final-normed readout, label logits.

There is no CPU fallback: importing works anywhere, but every call needs the built library and a B200; a missing
library raises `LayaLibraryMissing`.
"""
from .api import (Context, DecisionModel, DecisionOutput, BatchItem, ModelDesc, PackedMatrixQ8_0, Q8_0,
                  LayaError, LayaArgumentError, LayaOutOfRangeError, LayaNotSupportedError, LayaCudaError,
                  LayaNotFoundError, LayaDeviceTimeout, LayaLibraryMissing, lib, library_path, base_desc,
                  PRECISION_F32, PRECISION_Q8_0, Trainer, Batch, TrainingItem, TrainDesc, RlcdDesc, train_desc,
                  FORWARD_ACCURATE, FORWARD_BF16, Qwen35Model, Qwen35State, Qwen35Sequence, Qwen35Mark, DecoderDesc,
                  decoder_desc, DECODER_LINEAR,
                  DECODER_FULL, fit_temperatures, TemperatureFitDesc)

__all__ = ["Context", "DecisionModel", "DecisionOutput", "BatchItem", "ModelDesc", "PackedMatrixQ8_0", "Q8_0",
           "LayaError", "LayaArgumentError", "LayaOutOfRangeError", "LayaNotSupportedError", "LayaCudaError",
           "LayaNotFoundError", "LayaDeviceTimeout", "LayaLibraryMissing", "lib", "library_path", "base_desc",
           "PRECISION_F32", "PRECISION_Q8_0", "Trainer", "Batch", "TrainingItem", "TrainDesc", "RlcdDesc",
           "train_desc", "FORWARD_ACCURATE", "FORWARD_BF16", "Qwen35Model", "Qwen35State", "Qwen35Sequence", "Qwen35Mark",
           "DecoderDesc", "decoder_desc",
           "DECODER_LINEAR", "DECODER_FULL", "fit_temperatures", "TemperatureFitDesc"]
