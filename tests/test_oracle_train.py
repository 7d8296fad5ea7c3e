"""The training oracle against the reference's training fixtures and known answers (CPU only)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def tiny():
    from oracle.model import EncoderConfig
    g = json.load(open(os.path.join(GOLDEN, "training_tiny.json")))
    w = dict(np.load(os.path.join(GOLDEN, "training_tiny_model.npz")))
    cfg = EncoderConfig.from_hf(g["encoder_config"], head_layers=2, n_act=len(g["agent_config"]["act_costs"]) + 1)
    return cfg, w, g


def test_logits_and_every_gradient_match_pytorch():
    """TrainingGradientTests.LogitsMatchPyTorch / EveryGradientMatchesPyTorch (TrainingGradientTests.cs:44-85):
    logits within 1e-4, every gradient within 1e-4 of max |g|, nothing outside the loss gets a gradient."""
    import torch
    from oracle.train import TorchTrainModel
    cfg, w, g = tiny()
    m = TorchTrainModel(cfg, w)
    items = g["batch"]["items"]
    logits = m.forward(items, training=False)
    loss = sum((l * torch.tensor(it["coeff"], dtype=torch.float32)).sum() for l, it in zip(logits, items))
    loss.backward()
    for l, it in zip(logits, items):
        assert np.max(np.abs(l.detach().numpy() - np.array(it["logits"]))) < 1e-4
    want = dict(np.load(os.path.join(GOLDEN, "training_tiny_grads.npz")))
    got = m.grads()
    assert len(want) == 57
    for name, gw in want.items():
        rel = np.max(np.abs(got[name] - gw)) / max(np.max(np.abs(gw)), 1e-12)
        assert rel < 1e-4, f"{name}: {rel:.2e}"
    for name in got:
        if name.startswith("act_head."):
            assert not np.any(got[name])


def test_objective_matches_the_notebook():
    """TrainingTests.ObjectiveMatchesTheNotebookLossAndGradient (TrainingTests.cs:19-44)."""
    from oracle.train import rlcd
    _, _, g = tiny()
    o = g["objective"]
    loss, policy, ce, reward, grads = rlcd([np.array(l, np.float32) for l in o["logits"]],
                                           [np.array(t, np.float32) for t in o["target"]], o["qtypes"], o["sigma"],
                                           o["draws"])
    assert abs(ce - o["loss_ce"]) < 1e-5
    assert abs(policy - o["loss_rl"]) < 1e-4
    assert abs(reward - o["reward_mean"]) < 1e-4
    for gi, wi in zip(grads, o["grad"]):
        assert np.max(np.abs(gi - np.array(wi))) < 1e-4


def test_adamw_and_cosine_match_pytorch():
    """TrainingTests.AdamWAndTheCosineScheduleMatchPyTorch (TrainingTests.cs:46-70)."""
    from oracle.train import adamw_step, cosine_lr
    data = np.array([0.5, -1, 2, 0], np.float32)
    m = np.zeros(4, np.float32)
    v = np.zeros(4, np.float32)
    grads = [[0.1, -0.2, 0.3, 0], [0.5, 0.5, -0.5, 0], [-0.3, 0.1, 0.2, 1]]
    expected = [[0.39950001, -0.89900005, 1.898, 0], [0.3346217, -0.93149203, 1.91859365, 0],
                [0.32829964, -0.94257891, 1.9182955, -0.01597082]]
    rates = [0.07500025, 0.025000750000000013, 1e-6]
    lr = 0.1
    for step in range(3):
        adamw_step(data, np.array(grads[step], np.float32), m, v, step + 1, lr)
        lr = cosine_lr(0.1, step + 1, 3)
        assert np.allclose(data, expected[step], atol=1e-5)
        assert abs(lr - rates[step]) < 1e-9


def test_clipping_scales_to_the_maximum_norm():
    """TrainingTests.ClippingScalesToTheMaximumNorm (TrainingTests.cs:72-83)."""
    from oracle.train import clip_by_global_norm
    a = np.array([3, 0], np.float32)
    b = np.array([4], np.float32)
    assert abs(clip_by_global_norm([a, b], 1.0) - 5) < 1e-6
    assert abs(a[0] - 0.6) < 1e-5 and abs(b[0] - 0.8) < 1e-5


def test_dropout_hash_is_deterministic_and_fair():
    from oracle.train import dropout_mask, mix, uniform
    u = uniform(1234, np.arange(100000, dtype=np.uint64))
    assert u.min() >= 0 and u.max() < 1 and abs(u.mean() - 0.5) < 0.01
    assert np.array_equal(uniform(1234, np.arange(10, dtype=np.uint64)), u[:10])
    m = dropout_mask(100000, 0.1, mix(7, 3))
    assert abs((m == 0).mean() - 0.1) < 0.01


def test_temperature_fitting_recovers_a_known_temperature():
    """TrainingTests.TemperatureFittingRecoversAKnownTemperature (TrainingTests.cs:84-105): targets drawn from
    softmax(z / 2) are best explained by T = 2; five samples are too few (1); a type without samples gets 1.2."""
    from oracle.train import fit_one, fit_temperatures, softmax_f32
    rng = np.random.default_rng(5)
    samples = []
    for _ in range(400):
        z = (rng.random(4) * 8 - 4).astype(np.float32)
        samples.append((0, z, softmax_f32(z / np.float32(2))))
    assert abs(fit_one(samples) - 2.0) < 1e-3
    assert fit_one(samples[:5]) == 1.0
    by_type, by_bucket, counts = fit_temperatures(samples, 30)
    assert abs(by_type[0] - 2.0) < 1e-3 and by_type[2] == np.float32(1.2)
    assert abs(by_bucket["choice:3-5"] - 2.0) < 1e-3 and counts == {"choice:3-5": 400}
