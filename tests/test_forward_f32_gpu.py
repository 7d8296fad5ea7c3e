"""The decision forward's fp32-accurate path (LAYA_PRECISION_F32) on the B200: DecisionModel + ModernBertEncoder with
the reference's PackedMatrix products (DecisionModel.cs:50-99, ModernBertEncoder.Pack), here split bf16 products on
the tensor cores — weight hi (+ lo when the checkpoint is fp32) times activation hi + lo, fp32 accumulation — and fp16
attention.  A bf16 checkpoint (the reference's released checkpoints) takes two passes per product, an fp32 one three.

Bars (max |gpu − reference| / max |reference| per tensor, the north-star bar 2e-2 for floating-point results):
  * the training-tiny checkpoint end to end against the oracle's fp32 forward and against PyTorch's fp32 logits stored
    in the fixture;
  * ModernBERT-large geometry (config 4's encoder: h 1024, 16 heads, I 2624) with bf16 weights, teacher-forced layer
    by layer and end to end against the oracle;
  * batching and the device entry point bit-identical to singles and the host entry point.
"""
import numpy as np
import pytest

from conftest import max_rel
from test_forward_gpu import as_oracle_items, desc_for, tiny

pytestmark = pytest.mark.gpu
TOL = 2e-2
FP32_CLASS = 1e-3   # what this path actually holds against the fp32 oracle (measured ~1e-4 on logits, ~2e-5 per layer)


def to_bf16(x):
    """Round to nearest even on the top 16 bits; the values a bf16 checkpoint holds."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def test_tiny_checkpoint_fp32_forward(cuda, oracle_lib):
    """fp32 weights (three passes): option logits and action probabilities against the oracle and PyTorch."""
    import laya_b200
    from oracle.model import OracleModel
    cfg, w, g = tiny()
    model = laya_b200.DecisionModel(desc_for(cfg, max_tokens=1024, max_items=64, max_markers=256,
                                             precision=laya_b200.PRECISION_F32), w)
    items = [laya_b200.BatchItem(it["ids"], it["markers"], it["qtype"]) for it in g["batch"]["items"]]
    got = model.forward(items)
    want = OracleModel(cfg, w).forward(as_oracle_items(items))
    worst = 0.0
    for gi, (wl, wp), it in zip(got, want, g["batch"]["items"]):
        worst = max(worst, max_rel(gi.option_logits, wl))
        assert max_rel(gi.option_logits, wl) < TOL
        assert np.max(np.abs(gi.action_probabilities - wp)) < TOL
        assert max_rel(gi.option_logits, it["logits"]) < TOL
    print(f"tiny fp32: worst max rel against the oracle {worst:.2e}")
    assert worst < FP32_CLASS
    # the weights come back as hi + lo: within 2^-16 relative of what was uploaded
    name = "encoder.layers.1.attn.Wqkv.weight"
    back = model.ctx.download(name, w[name].shape)
    assert np.max(np.abs(back - w[name])) <= 2.0 ** -16 * np.max(np.abs(w[name]))
    model.ctx.close()


def test_tiny_checkpoint_bf16_weights(cuda, oracle_lib):
    """A bf16 checkpoint (two passes): uploaded as bf16 bits, against the oracle's fp32 forward of the same values;
    the projections read back exactly."""
    import laya_b200
    from oracle.model import OracleModel
    cfg, w, g = tiny()
    wb = {k: to_bf16(v) for k, v in w.items()}
    model = laya_b200.DecisionModel(desc_for(cfg, max_tokens=1024, max_items=64, max_markers=256,
                                             precision=laya_b200.PRECISION_F32), {})
    for name, arr in wb.items():
        if name != "temperature":
            model.ctx.upload(name, arr)
    items = [laya_b200.BatchItem(it["ids"], it["markers"], it["qtype"]) for it in g["batch"]["items"]]
    got = model.forward(items)
    want = OracleModel(cfg, wb).forward(as_oracle_items(items))
    for gi, (wl, wp) in zip(got, want):
        assert max_rel(gi.option_logits, wl) < TOL
        assert np.max(np.abs(gi.action_probabilities - wp)) < TOL
    name = "head.layers.0.linear1.weight"
    assert np.array_equal(model.ctx.download(name, wb[name].shape), wb[name])
    # batch = singles, bit for bit; run to run identical
    singles = [model.forward([it])[0] for it in items[:3]]
    again = model.forward(items)
    for a, b in zip(singles, got[:3]):
        assert np.array_equal(a.option_logits, b.option_logits)
    for a, b in zip(again, got):
        assert np.array_equal(a.option_logits, b.option_logits)
    model.ctx.close()


@pytest.fixture(scope="module")
def large(cuda, oracle_lib):
    import laya_b200
    from laya_b200 import workloads
    from oracle.model import EncoderConfig
    cfg = EncoderConfig(hidden=1024, intermediate=2624, layers=4, heads=16)
    w = {k: to_bf16(v) for k, v in workloads.training_weights(hidden=1024, intermediate=2624, layers=4,
                                                                 seed=3).items()}
    model = laya_b200.DecisionModel(desc_for(cfg, max_tokens=4096, max_items=16, max_markers=128,
                                             precision=laya_b200.PRECISION_F32), w)
    yield cfg, w, model
    model.ctx.close()


def test_large_geometry_layers_teacher_forced(large):
    """Each encoder layer (global 0 without attn_norm, sliding 1-2, global 3) on the oracle's input hidden states,
    segments of 512, 512 and a ragged 200."""
    from laya_b200 import workloads
    from oracle.model import OracleModel
    cfg, w, model = large
    om = OracleModel(cfg, w)
    items = workloads.decision_batch(rows=3, lengths=[512, 512, 200], seed=7, vocab=cfg.vocab)
    seg_len = np.array([len(it.token_ids) for it in items], np.int32)
    seg_start = np.concatenate([[0], np.cumsum(seg_len)[:-1]]).astype(np.int32)
    ids = np.concatenate([it.token_ids for it in items])
    h = om.ln(np.asarray(w["encoder.embeddings.tok_embeddings.weight"][ids], np.float32),
              "encoder.embeddings.norm.weight", None, cfg.norm_eps)
    for layer in range(cfg.layers):
        got = model.encoder_layer(layer, h, seg_len)
        want = om.encoder_layer(h, layer, seg_start, seg_len)
        err = max_rel(got, want)
        print(f"large layer {layer}: {err:.2e}")
        assert err < FP32_CLASS, f"layer {layer}: {err:.3e}"
        h = want


def test_large_geometry_end_to_end(large):
    from laya_b200 import workloads
    from oracle.model import OracleModel
    cfg, w, model = large
    items = workloads.decision_batch(rows=4, lengths=[512, 300, 77, 129], seed=8, vocab=cfg.vocab)
    got = model.forward(items)
    want = OracleModel(cfg, w).forward(as_oracle_items(items))
    for gi, (wl, wp) in zip(got, want):
        assert max_rel(gi.option_logits, wl) < TOL
        assert np.max(np.abs(gi.action_probabilities - wp)) < TOL
