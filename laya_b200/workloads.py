"""Seeded synthetic workloads for the hot path (no checkpoints or datasets exist on the GPU hosts).

Config 2 ("Q8_0 encoder inference"): ModernBERT-base geometry, every encoder and decision-head projection in Q8_0
(codes uniform in [-127, 127], block scales fp16(|N(0, scale)|), scale 0.002), embeddings fp32 N(0, 0.02), LayerNorm
γ = 1 and β = 0, biases 0, the small fp32 scorer / act head N(0, 0.02); a batch of 64 rows × 512 token ids uniform in
[5, 50368), all rows full length, five question kinds round-robin (choice-4, choice-6, score-4, noul, noul) with
option markers at j·⌊L/(k+1)⌋, j = 1..k.

Configs 1/3/4 (fine-tuning): every tensor N(0, 0.02) except LayerNorm γ = 1 and biases 0; rows of uniform token ids
in [5, vocab) with a per-row valid length (config 3: U{256..1024}), the same five question kinds, soft targets U(0, 1)
normalised per row, and the objective's standard-normal draws [groups, options].
"""
from typing import Dict, List, Tuple

import numpy as np

from .api import BatchItem, TrainingItem

# (qtype, options) of the five question kinds, assigned round-robin to rows
KINDS = [(0, 4), (0, 6), (1, 4), (2, 2), (2, 2)]


def q8_block(rng, n, k, scale):
    q = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    d = np.abs(rng.normal(0.0, scale, size=(n, k // 32))).astype(np.float16)
    return q, d


def decision_weights(hidden=768, intermediate=1152, layers=22, vocab=50368, head_layers=2, n_act=2, act_hidden=256,
                     q8_scale=0.002, seed=0) -> Tuple[Dict[str, np.ndarray], Dict[str, Tuple[np.ndarray, np.ndarray]]]:
    """fp32 tensors by safetensors name, and Q8_0 projections by name as (codes int8 [N, K], scales fp16 [N, K/32])."""
    rng = np.random.default_rng(seed)
    H, I = hidden, intermediate
    w: Dict[str, np.ndarray] = {}
    q8: Dict[str, Tuple[np.ndarray, np.ndarray]] = {}
    ones, zeros = (lambda n: np.ones(n, np.float32)), (lambda n: np.zeros(n, np.float32))
    w["encoder.embeddings.tok_embeddings.weight"] = rng.normal(0, 0.02, (vocab, H)).astype(np.float32)
    w["encoder.embeddings.norm.weight"] = ones(H)
    w["encoder.final_norm.weight"] = ones(H)
    for i in range(layers):
        p = f"encoder.layers.{i}."
        if i:
            w[p + "attn_norm.weight"] = ones(H)
        w[p + "mlp_norm.weight"] = ones(H)
        q8[p + "attn.Wqkv.weight"] = q8_block(rng, 3 * H, H, q8_scale)
        q8[p + "attn.Wo.weight"] = q8_block(rng, H, H, q8_scale)
        q8[p + "mlp.Wi.weight"] = q8_block(rng, 2 * I, H, q8_scale)
        q8[p + "mlp.Wo.weight"] = q8_block(rng, H, I, q8_scale)
    w["type_emb.weight"] = rng.normal(0, 0.02, (3, H)).astype(np.float32)
    for i in range(head_layers):
        p = f"head.layers.{i}."
        w[p + "norm1.weight"], w[p + "norm1.bias"] = ones(H), zeros(H)
        w[p + "norm2.weight"], w[p + "norm2.bias"] = ones(H), zeros(H)
        q8[p + "self_attn.in_proj_weight"] = q8_block(rng, 3 * H, H, q8_scale)
        w[p + "self_attn.in_proj_bias"] = zeros(3 * H)
        q8[p + "self_attn.out_proj.weight"] = q8_block(rng, H, H, q8_scale)
        w[p + "self_attn.out_proj.bias"] = zeros(H)
        q8[p + "linear1.weight"] = q8_block(rng, 4 * H, H, q8_scale)
        w[p + "linear1.bias"] = zeros(4 * H)
        q8[p + "linear2.weight"] = q8_block(rng, H, 4 * H, q8_scale)
        w[p + "linear2.bias"] = zeros(H)
    w["scorer.0.weight"], w["scorer.0.bias"] = ones(H), zeros(H)
    w["scorer.1.weight"] = rng.normal(0, 0.02, (H, H)).astype(np.float32)
    w["scorer.1.bias"] = zeros(H)
    w["scorer.3.weight"] = rng.normal(0, 0.02, (1, H)).astype(np.float32)
    w["scorer.3.bias"] = zeros(1)
    w["act_head.0.weight"] = rng.normal(0, 0.02, (act_hidden, H + 4)).astype(np.float32)
    w["act_head.0.bias"] = zeros(act_hidden)
    w["act_head.2.weight"] = rng.normal(0, 0.02, (n_act, act_hidden)).astype(np.float32)
    w["act_head.2.bias"] = zeros(n_act)
    return w, q8


def decision_batch(rows=64, length=512, vocab=50368, seed=1, lengths=None) -> List[BatchItem]:
    """Rows of uniform token ids in [5, vocab), question kinds round-robin, markers at j·⌊L/(k+1)⌋."""
    rng = np.random.default_rng(seed)
    items = []
    for r in range(rows):
        L = int(lengths[r]) if lengths is not None else length
        qt, k = KINDS[r % len(KINDS)]
        ids = rng.integers(5, vocab, size=L, dtype=np.int64)
        markers = [j * (L // (k + 1)) for j in range(1, k + 1)]
        items.append(BatchItem(ids, markers, qt))
    return items


def dequantized(q8):
    """Q8_0 projections as the oracle consumes them: (codes, scales as fp32 [N, K/32])."""
    return {k: (q, d.astype(np.float32)) for k, (q, d) in q8.items()}


def training_weights(hidden=768, intermediate=1152, layers=22, vocab=50368, head_layers=2, n_act=2, act_hidden=256,
                     std=0.02, seed=0) -> Dict[str, np.ndarray]:
    """fp32 tensors by safetensors name: N(0, std) weights, LayerNorm γ = 1, biases 0 (config 1/3/4)."""
    rng = np.random.default_rng(seed)
    H, I = hidden, intermediate
    w: Dict[str, np.ndarray] = {}
    ones, zeros = (lambda n: np.ones(n, np.float32)), (lambda n: np.zeros(n, np.float32))
    normal = lambda *shape: rng.normal(0, std, shape).astype(np.float32)
    w["encoder.embeddings.tok_embeddings.weight"] = normal(vocab, H)
    w["encoder.embeddings.norm.weight"] = ones(H)
    for i in range(layers):
        p = f"encoder.layers.{i}."
        if i:
            w[p + "attn_norm.weight"] = ones(H)
        w[p + "attn.Wqkv.weight"] = normal(3 * H, H)
        w[p + "attn.Wo.weight"] = normal(H, H)
        w[p + "mlp_norm.weight"] = ones(H)
        w[p + "mlp.Wi.weight"] = normal(2 * I, H)
        w[p + "mlp.Wo.weight"] = normal(H, I)
    w["encoder.final_norm.weight"] = ones(H)
    w["type_emb.weight"] = normal(3, H)
    for i in range(head_layers):
        p = f"head.layers.{i}."
        w[p + "norm1.weight"], w[p + "norm1.bias"] = ones(H), zeros(H)
        w[p + "self_attn.in_proj_weight"], w[p + "self_attn.in_proj_bias"] = normal(3 * H, H), zeros(3 * H)
        w[p + "self_attn.out_proj.weight"], w[p + "self_attn.out_proj.bias"] = normal(H, H), zeros(H)
        w[p + "norm2.weight"], w[p + "norm2.bias"] = ones(H), zeros(H)
        w[p + "linear1.weight"], w[p + "linear1.bias"] = normal(4 * H, H), zeros(4 * H)
        w[p + "linear2.weight"], w[p + "linear2.bias"] = normal(H, 4 * H), zeros(H)
    w["scorer.0.weight"], w["scorer.0.bias"] = ones(H), zeros(H)
    w["scorer.1.weight"], w["scorer.1.bias"] = normal(H, H), zeros(H)
    w["scorer.3.weight"], w["scorer.3.bias"] = normal(1, H), zeros(1)
    w["act_head.0.weight"], w["act_head.0.bias"] = normal(act_hidden, H + 4), zeros(act_hidden)
    w["act_head.2.weight"], w["act_head.2.bias"] = normal(n_act, act_hidden), zeros(n_act)
    return w


def training_batch(rows=32, min_len=256, max_len=1024, vocab=50368, seed=1000, groups=4):
    """(items, draws): rows with valid length U{min_len..max_len}, kinds round-robin, markers at j·⌊L/(k+1)⌋,
    targets U(0, 1) normalised, draws standard normal [groups, total options]."""
    rng = np.random.default_rng(seed)
    items = []
    for r in range(rows):
        L = int(rng.integers(min_len, max_len + 1))
        qt, k = KINDS[r % len(KINDS)]
        ids = rng.integers(5, vocab, size=L, dtype=np.int64)
        markers = np.array([j * (L // (k + 1)) for j in range(1, k + 1)], np.int64)
        t = rng.random(k).astype(np.float32)
        items.append(TrainingItem(ids, markers, qt, (t / t.sum()).astype(np.float32)))
    m = sum(it.options for it in items)
    draws = rng.standard_normal((groups, m))
    return items, draws


def mix(seed: int, salt: int) -> int:
    """Ops.Mix (Laya.Training/Ops.cs:236-241): the per-micro-step dropout seed Trainer.Train derives,
    Mix(Seed, microStep + 1) (Trainer.cs:129)."""
    m = (1 << 64) - 1
    z = (seed ^ ((salt * 0xD1B54A32D192ED03 + 0x8CB92BA72F3D8DD7) & m)) & m
    z = ((z ^ (z >> 33)) * 0xFF51AFD7ED558CCD) & m
    return z ^ (z >> 33)
