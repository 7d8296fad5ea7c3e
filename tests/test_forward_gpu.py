"""The batched decision forward on the B200 against the oracle, through the C ABI.

Bars (max |gpu - oracle| / max |oracle| per tensor):
  * stages and layers, teacher-forced (both sides start from the same input): 2e-2;
  * end-to-end logits of well-conditioned models: 2e-2 (the north-star bar for floating-point results);
  * run-to-run, batch-vs-singles and host-vs-device entry points: bit-identical.
The synthetic config-2 model (block scales |N(0, 0.002)|) is chaotic end to end: a 1e-6 relative nudge of its
embeddings already moves its logits by O(1) on the CPU oracle alone, so it is checked layer by layer (teacher forcing)
and its end-to-end run is checked on size-independent properties instead.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, bits, max_rel

pytestmark = pytest.mark.gpu
TOL = 2e-2


def tiny():
    from oracle.model import EncoderConfig
    g = json.load(open(os.path.join(GOLDEN, "training_tiny.json")))
    w = dict(np.load(os.path.join(GOLDEN, "training_tiny_model.npz")))
    cfg = EncoderConfig.from_hf(g["encoder_config"], head_layers=2, n_act=len(g["agent_config"]["act_costs"]) + 1)
    return cfg, w, g


def desc_for(cfg, **kw):
    import laya_b200
    kinds = [1 if cfg.kind(i) == "global" else 0 for i in range(cfg.layers)]
    d = dict(hidden=cfg.hidden, intermediate=cfg.intermediate, layers=cfg.layers, heads=cfg.heads, vocab=cfg.vocab,
             local_attention=cfg.local_attention, theta_global=cfg.theta_global, theta_local=cfg.theta_local,
             norm_eps=cfg.norm_eps, head_layers=cfg.head_layers, n_act=cfg.n_act, layer_kinds=kinds)
    d.update(kw)
    return laya_b200.base_desc(**d)


def as_oracle_items(items):
    from oracle.model import Item
    return [Item(np.asarray(it.token_ids), list(it.marker_positions), it.type) for it in items]


@pytest.fixture(scope="module")
def tiny_model(cuda):
    import laya_b200
    cfg, w, g = tiny()
    model = laya_b200.DecisionModel(desc_for(cfg, max_tokens=1024, max_items=64, max_markers=256), w)
    yield cfg, w, g, model
    model.ctx.close()


def tiny_oracle(cfg, w, oracle_lib):
    from oracle.model import OracleModel
    q8 = {}
    for name, arr in w.items():
        if (name.startswith("encoder.layers.") and name.endswith(("attn.Wqkv.weight", "attn.Wo.weight",
                                                                  "mlp.Wi.weight", "mlp.Wo.weight"))) or \
           (name.startswith("head.layers.") and name.endswith(("in_proj_weight", "out_proj.weight",
                                                               "linear1.weight", "linear2.weight"))):
            q8[name] = oracle_lib.q8_quantize_weights(arr)
    return OracleModel(cfg, w, q8)


def test_tiny_checkpoint_q8_forward_matches_oracle(tiny_model, oracle_lib):
    """The training-tiny checkpoint with every projection quantized to Q8_0 on the device (the PackedMatrixQ8_0
    constructor) against the oracle's Q8_0 forward: option logits and action probabilities."""
    import laya_b200
    cfg, w, g, model = tiny_model
    items = [laya_b200.BatchItem(it["ids"], it["markers"], it["qtype"]) for it in g["batch"]["items"]]
    got = model.forward(items)
    want = tiny_oracle(cfg, w, oracle_lib).forward(as_oracle_items(items))
    for gi, (wl, wp) in zip(got, want):
        assert max_rel(gi.option_logits, wl) < TOL
        assert np.max(np.abs(gi.action_probabilities - wp)) < TOL
    # and the Q8_0 model stays near PyTorch's fp32 logits (quantization moves them by a few percent at most)
    for gi, it in zip(got, g["batch"]["items"]):
        assert max_rel(gi.option_logits, it["logits"]) < 0.1


def test_device_packed_weights_equal_the_oracle_quantizer(tiny_model, oracle_lib):
    cfg, w, g, model = tiny_model
    for name in ["encoder.layers.1.attn.Wqkv.weight", "encoder.layers.2.mlp.Wi.weight", "head.layers.0.linear2.weight"]:
        q, d = oracle_lib.q8_quantize_weights(w[name])
        deq = model.ctx.download(name, w[name].shape)
        assert np.array_equal(deq, q.astype(np.float32) * np.repeat(d, 32, axis=1))


def test_batch_equals_singles_and_is_deterministic(tiny_model):
    """DecisionModel.Forward over a batch is identical to one question at a time (DecisionModel.cs:117-124)."""
    import laya_b200
    cfg, w, g, model = tiny_model
    rng = np.random.default_rng(3)
    items = []
    for L in [1, 7, 64, 65, 130, 200]:
        k = int(rng.integers(1, 5))
        items.append(laya_b200.BatchItem(rng.integers(3, cfg.vocab, L), sorted(rng.integers(0, L, k).tolist()),
                                         int(rng.integers(0, 3))))
    batch = model.forward(items)
    again = model.forward(items)
    for a, b in zip(batch, again):
        assert np.array_equal(bits(a.option_logits), bits(b.option_logits))
    for it, b in zip(items, batch):
        s = model.forward([it])[0]
        assert np.array_equal(bits(s.option_logits), bits(b.option_logits))
        assert np.array_equal(bits(s.action_probabilities), bits(b.action_probabilities))


def test_ragged_segments_match_oracle(tiny_model, oracle_lib):
    """Segments of 1..300 tokens, windows wider than the segment, single-token segments, markers at 0 and at the end."""
    import laya_b200
    cfg, w, g, model = tiny_model
    rng = np.random.default_rng(4)
    items = []
    for L in [1, 2, 9, 63, 64, 65, 127, 128, 129, 300]:
        k = int(rng.integers(1, 6))
        m = sorted(set([0, L - 1] + rng.integers(0, L, k).tolist()))
        items.append(laya_b200.BatchItem(rng.integers(3, cfg.vocab, L), m, int(rng.integers(0, 3))))
    got = model.forward(items)
    want = tiny_oracle(cfg, w, oracle_lib).forward(as_oracle_items(items))
    for gi, (wl, wp) in zip(got, want):
        assert max_rel(gi.option_logits, wl) < TOL


def test_errors_are_reported_like_the_reference(tiny_model):
    """Token ids outside the vocabulary -> ArgumentOutOfRangeException (ModernBertEncoder.cs:136-139); markers past
    the question and oversized batches are rejected before anything runs."""
    import laya_b200
    cfg, w, g, model = tiny_model
    with pytest.raises(laya_b200.LayaOutOfRangeError):
        model.forward([laya_b200.BatchItem([5, cfg.vocab], [0], 0)])
    with pytest.raises(laya_b200.LayaOutOfRangeError):
        model.forward([laya_b200.BatchItem([5, 6, 7], [3], 0)])
    with pytest.raises(laya_b200.LayaArgumentError):
        model.forward([laya_b200.BatchItem(np.full(2000, 5), [0], 0)])
    # the context stays usable
    ok = model.forward([laya_b200.BatchItem([5, 6, 7], [1], 0)])
    assert np.isfinite(ok[0].option_logits).all()


# ------------------------------------------------------------------------------------------------ config-2 geometry
@pytest.fixture(scope="module")
def base_q8(cuda):
    """ModernBERT-base geometry, 3 encoder layers (global, sliding, sliding), synthetic Q8_0 weights of config 2."""
    import laya_b200
    from laya_b200 import workloads
    from oracle.model import EncoderConfig
    cfg = EncoderConfig(layers=3)
    w, q8 = workloads.decision_weights(layers=3, seed=0)
    model = laya_b200.DecisionModel(desc_for(cfg, max_tokens=4096, max_items=16, max_markers=128), w, q8)
    yield cfg, w, q8, model
    model.ctx.close()


def test_config2_layers_teacher_forced(base_q8, oracle_lib):
    """Each encoder layer of the config-2 model on the same input hidden states (global layer 0 without attn_norm,
    sliding layers 1-2), 2 segments × 512 + a ragged 200: within 2e-2 of the oracle per layer."""
    from laya_b200 import workloads
    from oracle.model import OracleModel
    cfg, w, q8, model = base_q8
    om = OracleModel(cfg, w, workloads.dequantized(q8))
    items = workloads.decision_batch(rows=3, lengths=[512, 512, 200], seed=7)
    seg_len = np.array([len(it.token_ids) for it in items], np.int32)
    seg_start = np.concatenate([[0], np.cumsum(seg_len)[:-1]]).astype(np.int32)
    ids = np.concatenate([it.token_ids for it in items])
    h = om.ln(np.asarray(w["encoder.embeddings.tok_embeddings.weight"][ids], np.float32),
              "encoder.embeddings.norm.weight", None, cfg.norm_eps)
    for layer in range(cfg.layers):
        got = model.encoder_layer(layer, h, seg_len)
        want = om.encoder_layer(h, layer, seg_start, seg_len)
        err = max_rel(got, want)
        assert err < TOL, f"layer {layer}: {err:.3e}"
        h = want


def test_conditioned_config2_end_to_end(cuda, oracle_lib):
    """Config-2 geometry with block scales |N(0, 0.0002)| (a well-conditioned model): logits end to end."""
    import laya_b200
    from laya_b200 import workloads
    from oracle.model import EncoderConfig, OracleModel
    cfg = EncoderConfig(layers=4)
    w, q8 = workloads.decision_weights(layers=4, seed=2, q8_scale=0.0002)
    model = laya_b200.DecisionModel(desc_for(cfg, max_tokens=4096, max_items=16, max_markers=128), w, q8)
    items = workloads.decision_batch(rows=5, lengths=[512, 300, 77, 512, 129], seed=8)
    got = model.forward(items)
    want = OracleModel(cfg, w, workloads.dequantized(q8)).forward(as_oracle_items(items))
    model.ctx.close()
    for gi, (wl, wp) in zip(got, want):
        assert max_rel(gi.option_logits, wl) < TOL
        assert np.max(np.abs(gi.action_probabilities - wp)) < TOL


def test_config2_full_forward_properties(cuda):
    """The full config-2 workload (22 layers, 64 × 512): finite logits, probabilities summing to one, the device
    entry point equal to the host one bit for bit, and identical results run to run."""
    import laya_b200
    from laya_b200 import workloads
    torch = cuda
    w, q8 = workloads.decision_weights(seed=0)
    model = laya_b200.DecisionModel(laya_b200.base_desc(max_tokens=32768, max_items=64, max_markers=512), w, q8)
    items = workloads.decision_batch(rows=64, length=512, seed=1)
    a = model.forward(items)
    b = model.forward(items)
    for x, y in zip(a, b):
        assert np.isfinite(x.option_logits).all()
        assert abs(float(x.action_probabilities.sum()) - 1) < 1e-5
        assert np.array_equal(bits(x.option_logits), bits(y.option_logits))
    ids, seg_len, qtype, counts, markers = model.pack(items)
    dev = [torch.from_numpy(v).cuda() for v in (ids, seg_len, qtype, counts, markers)]
    logits = torch.zeros(int(counts.sum()), dtype=torch.float32, device="cuda")
    act = torch.zeros(len(items) * 2, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    laya_b200.api.check(laya_b200.lib().laya_decision_forward_device(
        model.ctx.handle, dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), len(items), int(ids.size),
        dev[3].data_ptr(), dev[4].data_ptr(), int(counts.sum()), logits.data_ptr(), act.data_ptr()))
    model.ctx.synchronize()
    want = np.concatenate([x.option_logits for x in a])
    assert np.array_equal(bits(logits.cpu().numpy()), bits(want))
    model.ctx.close()
