"""The CPU oracle against the reference's own golden vectors and known answers (CPU only).

Each test names the reference test it restates (tests/StructuredDecisions.Tests/..., inside the reference project).
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, max_rel


def test_quantizers_round_as_ggml_does(oracle_lib):
    """PackedMatrixQ8_0Tests.QuantizersRoundAsGgmlDoes (PackedMatrixQ8_0Tests.cs:12-44)."""
    o = oracle_lib
    x = np.zeros(32, np.float32)
    x[:6] = [127, 2.5, -2.5, 3.5, -0.5, 126.49]
    d, q = o.q8_quantize_weight_block(x)
    assert d == 1.0
    assert list(q[:6]) == [127, 3, -3, 4, -1, 126]
    qa, da = o.q8_quantize_activations(x[None])
    assert da[0, 0] == 1.0
    assert list(qa[0, :6]) == [127, 2, -2, 4, 0, 126]
    assert np.all(qa[0, 6:] == 0)
    x[:] = 0
    x[0] = 1
    d, q = o.q8_quantize_weight_block(x)
    assert d == np.float32(np.float16(1 / 127)) and d != np.float32(1 / 127)
    x[:] = 0
    d, q = o.q8_quantize_weight_block(x)
    assert d == 0 and np.all(q == 0)


def test_one_matmul_matches_torch_as_ggml(oracle_lib):
    """Qwen35ParityTests.Q8_0MatchesTransformersComputingAsGgml, the single-matmul part (Qwen35ParityTests.cs:118-125):
    within 1e-6 of torch's ggml emulation, on inputs with exact half steps."""
    f = np.load(os.path.join(GOLDEN, "q8_matmul.npz"))
    qw, dw = oracle_lib.q8_quantize_weights(f["w"])
    y = oracle_lib.q8_linear(f["x"], qw, dw)
    rel = np.linalg.norm(y - f["y"]) / np.linalg.norm(f["y"])
    assert rel < 1e-6


def test_q8_is_close_to_fp32_product(oracle_lib):
    """PackedMatrixQ8_0Tests.IsCloseToTheFp32Product (PackedMatrixQ8_0Tests.cs:102-120)."""
    rng = np.random.default_rng(3)
    w = (rng.random((192, 2560)) * 2 - 1).astype(np.float32)
    x = (rng.random((9, 2560)) * 2 - 1).astype(np.float32)
    exact = oracle_lib.linear_f32(x, w)
    qw, dw = oracle_lib.q8_quantize_weights(w)
    quant = oracle_lib.q8_linear(x, qw, dw)
    rel = np.sqrt(np.sum((exact - quant) ** 2.0) / np.sum(exact ** 2.0))
    assert 1e-4 <= rel <= 1e-2


def test_dequantize_within_half_a_step(oracle_lib):
    """PackedMatrixQ8_0Tests.DequantizeIsWithinHalfAStep (PackedMatrixQ8_0Tests.cs:126-143)."""
    rng = np.random.default_rng(5)
    w = (rng.random((70, 64)) * 2 - 1).astype(np.float32)
    q, d = oracle_lib.q8_quantize_weights(w)
    deq = q.astype(np.float32) * np.repeat(d, 32, axis=1)
    for b in range(2):
        blk = w[:, b * 32:(b + 1) * 32]
        step = np.abs(blk).max(1).astype(np.float32) / np.float32(127)
        step = step.astype(np.float16).astype(np.float32)
        assert np.all(np.abs(deq[:, b * 32:(b + 1) * 32] - blk) <= step[:, None] * (0.5 + 127 / 2048) + 1e-7)


def test_block_dots_are_exact_integers(oracle_lib):
    """The int32 block dots the Q8_0 product is built from equal an int64 numpy computation."""
    rng = np.random.default_rng(11)
    qx = rng.integers(-127, 128, (13, 96), dtype=np.int8)
    qw = rng.integers(-127, 128, (40, 96), dtype=np.int8)
    dots = oracle_lib.q8_block_dots(qx, qw)
    want = np.einsum("rbk,nbk->rnb", qx.reshape(13, 3, 32).astype(np.int64), qw.reshape(40, 3, 32).astype(np.int64))
    assert np.array_equal(dots, want)


@pytest.mark.parametrize("x,expected", [(0.0, 0.0), (1.0, 0.8413447), (-1.0, -0.15865529), (3.0, 2.9959502),
                                        (-3.0, -0.00404969)])
def test_gelu_is_the_exact_erf_form(oracle_lib, x, expected):
    """NumericsTests.GeluIsTheExactErfForm (NumericsTests.cs:156-167)."""
    assert abs(float(oracle_lib.gelu(np.array([x], np.float32))[0]) - expected) < 5e-6


def test_vector_exp_matches_the_library(oracle_lib):
    """NumericsTests.VectorExpMatchesTheLibraryCall (NumericsTests.cs:169-181)."""
    L = oracle_lib.lib()
    for x in np.arange(-87.0, 88.0, 0.37):
        got = L.lo_exp_vec(np.float32(x))
        want = np.exp(np.float32(x), dtype=np.float32)
        assert abs(got - want) <= max(abs(want) * 2e-6, 1.4e-45)


def test_erf_is_accurate(oracle_lib):
    """NumericsTests.ErfIsAccurateAcrossTheRange (NumericsTests.cs:211-220), on the vector form the hot path uses."""
    L = oracle_lib.lib()
    for x, e in [(0.0, 0.0), (0.25, 0.2763263902), (0.5, 0.5204998778), (1.0, 0.8427007929), (2.0, 0.9953222650),
                 (3.0, 0.9999779095), (-1.5, -0.9661051465)]:
        assert abs(L.lo_erf_vec(np.float32(x)) - e) < 3e-6


def _tiny():
    from oracle.model import EncoderConfig, Item
    g = json.load(open(os.path.join(GOLDEN, "training_tiny.json")))
    w = dict(np.load(os.path.join(GOLDEN, "training_tiny_model.npz")))
    cfg = EncoderConfig.from_hf(g["encoder_config"], head_layers=2, n_act=len(g["agent_config"]["act_costs"]) + 1)
    items = [Item(np.array(it["ids"]), it["markers"], it["qtype"]) for it in g["batch"]["items"]]
    return cfg, w, items, g


def test_fp32_forward_matches_pytorch_logits(oracle_lib):
    """TrainingGradientTests' logit check (TrainingGradientTests.cs:44-56): the fp32 forward of the training-tiny
    checkpoint reproduces PyTorch's logits within 1e-4."""
    from oracle.model import OracleModel
    cfg, w, items, g = _tiny()
    out = OracleModel(cfg, w).forward(items)
    for (logits, probs), it in zip(out, g["batch"]["items"]):
        assert np.max(np.abs(logits - np.array(it["logits"], np.float32))) < 1e-4
        assert abs(probs.sum() - 1) < 1e-5


def test_batch_equals_singles(oracle_lib):
    """Concatenating questions is the same as running them one at a time (DecisionModel.cs:117-124)."""
    from oracle.model import OracleModel
    cfg, w, items, _ = _tiny()
    m = OracleModel(cfg, w)
    batch = m.forward(items)
    for it, (bl, bp) in zip(items, batch):
        sl, sp = m.forward([it])[0]
        assert np.array_equal(bl, sl) and np.array_equal(bp, sp)
