"""The fine-tuning step at the sizes the benchmark configurations state, against the training oracle.

  * config 1 in full: ModernBERT-base, all 22 layers, the full 50 368-token vocabulary, N(0, 0.02) weights from seed 0,
    8 rows of valid length U{64..256}, dropout off; logits, every parameter gradient, then one clipped AdamW step on
    the device's own gradients bit-compared with AdamW.Step's fp32 arithmetic (AdamW.cs:29-73, 103-130);
  * config 4's row length: ModernBERT-large widths on two layers (global, then sliding ±64) with an 8192-token row —
    the global backward over 64 key tiles and window skipping far from the row start (Ops.cs:329-438);
  * config 3's row length: ModernBERT-base widths on two layers with rows of the full 1024 tokens.

Bars: logits max |gpu − oracle| / max |oracle| ≤ 2e-2 per item; every gradient tensor cosine ≥ 0.999 and max
|gpu − oracle| / max |oracle| ≤ 2e-2, elementwise.  Stated exceptions (normwise ≤ 2e-2 instead of elementwise):
the decision head's linear1 weight and bias of each head layer, and its second LayerNorm (norm2) of each head
layer.  Their pre-activations include values within ~1e-6 of zero; the GPU forward (fp32-accurate hi/lo products,
~2^-16 relative) and the oracle's fp32 forward disagree on the sign of a handful of those, and each flipped ReLU
mask bit moves one whole row of linear1's gradient (and, through it, norm2's) by a few percent of that tensor's
largest element while leaving its cosine at 0.9999.
"""
import numpy as np
import pytest

from conftest import max_rel

pytestmark = pytest.mark.gpu
TOL = 2e-2
COS = 0.999
# tensors held to the normwise relative bar (the module docstring gives the reason)
RELU_ROWS = ("linear1.weight", "linear1.bias", "norm2.weight", "norm2.bias")


def _cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / max(na * nb, 1e-300))


def _norm_rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def _check(t, want, skip_prefix=("act_head.",)):
    """Every gradient against the oracle's; returns the per-tensor figures for the failure message."""
    bad, rows = [], []
    for name, gw in want.items():
        if name.startswith(skip_prefix):
            continue
        got = t.gradient(name, gw.shape)
        c = _cosine(got, gw)
        normwise = name.startswith("head.layers.") and name.endswith(RELU_ROWS)
        r = (_norm_rel if normwise else max_rel)(got, gw)
        rows.append((name, c, r))
        if c < COS or r > TOL:
            bad.append(f"{name}: cos {c:.6f} {'norm' if normwise else 'max'}-rel {r:.3e}")
    assert not bad, bad
    return rows


def _desc(cfg, **kw):
    import laya_b200
    kinds = [1 if cfg.kind(i) == "global" else 0 for i in range(cfg.layers)]
    d = dict(hidden=cfg.hidden, intermediate=cfg.intermediate, layers=cfg.layers, heads=cfg.heads, vocab=cfg.vocab,
             local_attention=cfg.local_attention, theta_global=cfg.theta_global, theta_local=cfg.theta_local,
             norm_eps=cfg.norm_eps, head_layers=cfg.head_layers, n_act=cfg.n_act, layer_kinds=kinds)
    d.update(kw)
    return laya_b200.base_desc(**d)


def _oracle(cfg, w, items, seed):
    """The oracle's logits and gradients of Σ coeff · logits for standard-normal coefficients."""
    import torch
    from oracle.train import TorchTrainModel
    m = TorchTrainModel(cfg, w, head_dropout=0.0)
    oi = [{"ids": it.token_ids, "markers": list(it.marker_positions), "qtype": it.question_type} for it in items]
    ref = m.forward(oi, training=False)
    rng = np.random.default_rng(seed)
    coeff = [rng.standard_normal(it.options).astype(np.float32) for it in items]
    sum((r * torch.from_numpy(c)).sum() for r, c in zip(ref, coeff)).backward()
    return [r.detach().numpy() for r in ref], coeff, m.grads()


def _step(cfg, w, items, seed, max_tokens, max_segment):
    import laya_b200
    lo, coeff, grads = _oracle(cfg, w, items, seed)
    t = laya_b200.Trainer(_desc(cfg, max_tokens=max_tokens, max_items=len(items), max_markers=8 * len(items)),
                          laya_b200.train_desc(max_segment=max_segment))
    t.load(w)
    b = t.batch(items)
    t.zero_grads()
    logits = t.forward(b, training=False)
    for l, r in zip(logits, lo):
        assert max_rel(l, r) <= TOL, (l, r)
    t.backward(b, coeff)
    return t, b, grads


def test_config1_full_model(cuda):
    """Config 1 as stated: the whole 22-layer ModernBERT-base with its vocabulary, 8 rows of U{64..256} tokens;
    logits and all gradients, then one clipped AdamW step bit for bit."""
    from laya_b200.workloads import training_batch, training_weights
    from oracle.model import EncoderConfig
    from oracle.train import adamw_step
    cfg = EncoderConfig()
    w = training_weights(seed=0)
    items, _ = training_batch(rows=8, min_len=64, max_len=256, seed=0)
    T = sum(len(it.token_ids) for it in items)
    t, b, want = _step(cfg, w, items, seed=1, max_tokens=T, max_segment=256)
    _check(t, want)
    # one clipped AdamW step (lr 2e-5, the config's rate) on the device's own gradients
    names = t.names()
    params = {n: t.download(n, (r, c)).ravel() for n, r, c in names}
    grads = {n: t.gradient(n, (r, c)).ravel() for n, r, c in names}
    t.set_lr(2e-5, 2e-5)
    norm = t.clip_and_step(max_norm=1.0)
    want_norm = float(np.sqrt(sum(np.sum(g.astype(np.float64) ** 2) for g in grads.values())))
    assert abs(norm - want_norm) <= 1e-9 * want_norm
    coef = 1.0 / (norm + 1e-6)          # ClipByGlobalNorm scales only when this is below 1
    for n, r, c in names:
        p = params[n].copy()
        g = grads[n] * np.float32(coef) if coef < 1.0 else grads[n]
        adamw_step(p, g, np.zeros_like(p), np.zeros_like(p), 1, 2e-5)
        got = t.download(n, (r, c)).ravel()
        assert np.array_equal(got.view(np.uint32), p.view(np.uint32)), n
    b.close()
    t.close()


def test_config4_row_length(cuda):
    """ModernBERT-large widths (hidden 1024, 16 heads × 64, GeGLU 2624) on a global and a sliding layer with an
    8192-token row beside a 1024-token one: logits and every gradient."""
    from laya_b200.workloads import training_batch, training_weights
    from oracle.model import EncoderConfig
    cfg = EncoderConfig(hidden=1024, intermediate=2624, layers=2, heads=16, vocab=3000)
    w = training_weights(hidden=1024, intermediate=2624, layers=2, vocab=3000, seed=21)
    long_row, _ = training_batch(rows=1, min_len=8192, max_len=8192, vocab=3000, seed=22)
    short_row, _ = training_batch(rows=1, min_len=1024, max_len=1024, vocab=3000, seed=23)
    items = long_row + short_row
    t, b, want = _step(cfg, w, items, seed=24, max_tokens=8192 + 1024, max_segment=8192)
    _check(t, want)
    b.close()
    t.close()


def test_config3_row_length(cuda):
    """ModernBERT-base widths on a global and a sliding layer with rows of config 3's full 1024 tokens (and two
    shorter ones): logits and every gradient."""
    from laya_b200.api import TrainingItem
    from laya_b200.workloads import training_batch, training_weights
    from oracle.model import EncoderConfig
    cfg = EncoderConfig(layers=2, vocab=3000)
    w = training_weights(layers=2, vocab=3000, seed=31)
    full, _ = training_batch(rows=2, min_len=1024, max_len=1024, vocab=3000, seed=32)
    rest, _ = training_batch(rows=2, min_len=256, max_len=1023, vocab=3000, seed=33)
    items = full + rest
    assert all(isinstance(it, TrainingItem) for it in items)
    T = sum(len(it.token_ids) for it in items)
    t, b, want = _step(cfg, w, items, seed=34, max_tokens=T, max_segment=1024)
    _check(t, want)
    b.close()
    t.close()
