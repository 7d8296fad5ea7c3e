"""Seeded synthetic workloads for the hot path (no checkpoints or datasets exist on the GPU hosts).

Config 2 ("Q8_0 encoder inference"): ModernBERT-base geometry, every encoder and decision-head projection in Q8_0
(codes uniform in [-127, 127], block scales fp16(|N(0, scale)|), scale 0.002), embeddings fp32 N(0, 0.02), LayerNorm
γ = 1 and β = 0, biases 0, the small fp32 scorer / act head N(0, 0.02); a batch of 64 rows × 512 token ids uniform in
[5, 50368), all rows full length, five question kinds round-robin (choice-4, choice-6, score-4, noul, noul) with
option markers at j·⌊L/(k+1)⌋, j = 1..k.

Configs 1/3/4 (fine-tuning): every tensor N(0, 0.02) except LayerNorm γ = 1 and biases 0; rows of uniform token ids
in [5, vocab) with a per-row valid length (config 3: U{256..1024}), the same five question kinds, soft targets U(0, 1)
normalised per row, and the objective's standard-normal draws [groups, options].

Config 5 (Mica hybrid decoder prefill): Qwen3.5 geometry (32 layers of [DeltaNet ×3, full ×1], h 2560, I 9216,
vocab 151936); projections and the tied token table in Q8_0 (codes uniform in [-127, 127], block scales
fp16(|N(0, scale)|)), norms, conv taps N(0, 0.02), A_log ~ U(0, 2), dt_bias 0; 8 rows × 2048 token ids uniform in
[0, vocab), 26 label ids.  `decoder_weights` gives the same tensors in fp32 (N(0, std) projections) for parity cases.
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


def bf16_checkpoint_weights(hidden=1024, intermediate=2624, layers=28, vocab=50368, head_layers=2, n_act=2,
                            act_hidden=256, std=0.02, seed=0, **_) -> Dict[str, np.ndarray]:
    """The tensors of training_weights' names and shapes as a bf16 checkpoint holds them: N(0, std) draws truncated
    to bf16 values (returned as fp32), LayerNorm γ = 1, biases 0.  float32 draws, so a 400M-parameter model is made
    in seconds."""
    rng = np.random.default_rng(seed)
    shapes = {k: v.shape for k, v in training_weights(hidden=8, intermediate=8, layers=layers, vocab=8, head_layers=head_layers,
                                                      n_act=n_act, act_hidden=8, seed=0).items()}
    out: Dict[str, np.ndarray] = {}
    H, I = hidden, intermediate
    real = {"encoder.embeddings.tok_embeddings.weight": (vocab, H), "type_emb.weight": (3, H),
            "scorer.3.weight": (1, H), "scorer.3.bias": (1,), "act_head.0.weight": (act_hidden, H + 4),
            "act_head.0.bias": (act_hidden,), "act_head.2.weight": (n_act, act_hidden), "act_head.2.bias": (n_act,)}
    for name in shapes:
        if name in real:
            shape = real[name]
        elif name.endswith(("attn.Wqkv.weight", "self_attn.in_proj_weight")):
            shape = (3 * H, H)
        elif name.endswith("self_attn.in_proj_bias"):
            shape = (3 * H,)
        elif name.endswith("mlp.Wi.weight"):
            shape = (2 * I, H)
        elif name.endswith("mlp.Wo.weight"):
            shape = (H, I)
        elif name.endswith("linear1.weight"):
            shape = (4 * H, H)
        elif name.endswith("linear1.bias"):
            shape = (4 * H,)
        elif name.endswith("linear2.weight"):
            shape = (H, 4 * H)
        elif name.endswith((".weight", ".bias")) and len(shapes[name]) == 2:
            shape = (H, H)
        else:
            shape = (H,)
        if name.endswith("bias"):
            out[name] = np.zeros(shape, np.float32)
        elif len(shape) == 1:
            out[name] = np.ones(shape, np.float32)
        else:
            x = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
            out[name] = (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    return out


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


# ----------------------------------------------------------------------------------------------- Mica decoder
MICA_KINDS = (["linear"] * 3 + ["full"]) * 8
MICA = dict(hidden=2560, intermediate=9216, vocab=151936, heads=16, kv_heads=4, head_dim=128, lin_k_heads=16,
            lin_v_heads=16, lin_k_dim=128, lin_v_dim=128, conv_kernel=4)


def decoder_shapes(kinds, hidden, intermediate, vocab, heads, kv_heads, head_dim, lin_k_heads, lin_v_heads,
                   lin_k_dim, lin_v_dim, conv_kernel):
    """(name, shape, kind) of every checkpoint tensor of a Qwen3.5 text decoder; kind is "proj" (a Q8_0 projection
    or the token table), "norm", "conv", "A_log", "dt_bias"."""
    kd, vd = lin_k_heads * lin_k_dim, lin_v_heads * lin_v_dim
    cd = 2 * kd + vd
    out = [("model.embed_tokens.weight", (vocab, hidden), "proj"), ("model.norm.weight", (hidden,), "norm")]
    for i, k in enumerate(kinds):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", (hidden,), "norm"),
                (p + "post_attention_layernorm.weight", (hidden,), "norm"),
                (p + "mlp.gate_proj.weight", (intermediate, hidden), "proj"),
                (p + "mlp.up_proj.weight", (intermediate, hidden), "proj"),
                (p + "mlp.down_proj.weight", (hidden, intermediate), "proj")]
        if k == "full":
            a = p + "self_attn."
            out += [(a + "q_proj.weight", (2 * heads * head_dim, hidden), "proj"),
                    (a + "k_proj.weight", (kv_heads * head_dim, hidden), "proj"),
                    (a + "v_proj.weight", (kv_heads * head_dim, hidden), "proj"),
                    (a + "o_proj.weight", (hidden, heads * head_dim), "proj"),
                    (a + "q_norm.weight", (head_dim,), "norm"), (a + "k_norm.weight", (head_dim,), "norm")]
        else:
            a = p + "linear_attn."
            out += [(a + "in_proj_qkv.weight", (cd, hidden), "proj"), (a + "in_proj_z.weight", (vd, hidden), "proj"),
                    (a + "in_proj_b.weight", (lin_v_heads, hidden), "proj"),
                    (a + "in_proj_a.weight", (lin_v_heads, hidden), "proj"),
                    (a + "out_proj.weight", (hidden, vd), "proj"), (a + "conv1d.weight", (cd, 1, conv_kernel), "conv"),
                    (a + "A_log", (lin_v_heads,), "A_log"), (a + "dt_bias", (lin_v_heads,), "dt_bias"),
                    (a + "norm.weight", (lin_v_dim,), "gnorm")]
    return out


def _vector(rng, shape, kind):
    if kind == "A_log":
        return rng.uniform(0.0, 2.0, shape).astype(np.float32)
    if kind == "dt_bias":
        return np.zeros(shape, np.float32)
    if kind == "gnorm":
        return (1.0 + rng.normal(0.0, 0.02, shape)).astype(np.float32)
    return rng.normal(0.0, 0.02, shape).astype(np.float32)


def decoder_weights(kinds, seed=0, std=0.02, **geometry) -> Dict[str, np.ndarray]:
    """Every tensor in fp32 (projections N(0, std)), for parity cases small enough for the CPU oracle."""
    g = dict(MICA)
    g.update(geometry)
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape, kind in decoder_shapes(kinds, **g):
        w[name] = rng.normal(0.0, std, shape).astype(np.float32) if kind == "proj" else _vector(rng, shape, kind)
    return w


def decoder_q8_weights(kinds, seed=0, q8_scale=0.0004, **geometry):
    """(Q8_0 projections {name: (int8 codes [N, K], fp16 scales [N, K/32])}, fp32 vectors {name: array}).  The codes
    of every projection are windows of one seeded pool of random bytes, so a 4-billion-parameter model is made in
    seconds."""
    g = dict(MICA)
    g.update(geometry)
    rng = np.random.default_rng(seed)
    shapes = decoder_shapes(kinds, **g)
    largest = max(int(np.prod(s)) for _, s, k in shapes if k == "proj")
    pool = rng.integers(-127, 128, size=largest + 65537, dtype=np.int8)
    scales = np.abs(rng.normal(0.0, q8_scale, size=largest // 32 + 4097)).astype(np.float16)
    q8, vec = {}, {}
    for name, shape, kind in shapes:
        if kind == "proj":
            n, k = shape
            o = int(rng.integers(0, 65536))
            so = int(rng.integers(0, 4096))
            q8[name] = (pool[o:o + n * k].reshape(n, k), scales[so:so + n * k // 32].reshape(n, k // 32))
        else:
            vec[name] = _vector(rng, shape, kind)
    return q8, vec


def decoder_batch(rows=8, length=2048, vocab=151936, n_labels=26, seed=5):
    """rows × length token ids uniform in [0, vocab) and n_labels distinct label ids."""
    rng = np.random.default_rng(seed)
    seqs = [rng.integers(0, vocab, size=length).astype(np.int32) for _ in range(rows)]
    labels = rng.choice(vocab, size=n_labels, replace=False).astype(np.int32)
    return seqs, labels
