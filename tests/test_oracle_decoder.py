"""The decoder oracle (oracle/decoder.py) against the reference's qwen35-tiny fixture (CPU only).

The bars are Qwen35ParityTests' own (Qwen35ParityTests.cs:45-136), with its relative error ||a - b|| / ||b||:
  * fp32 products: every recorded state and the logits within 1e-4 of transformers' fp32 run, and no further from the
    fp64 run than 2 × transformers' own fp32 error + 1e-7;
  * Q8_0 products (as ggml computes them): every state within 0.2 × of what Q8_0 moves it from the exact model, the
    first mixer within 1e-4, the logits within 0.2 ×.
"""
import numpy as np
import pytest

from conftest import GOLDEN


def rel(expected, actual):
    e = np.asarray(expected, np.float64).ravel()
    a = np.asarray(actual, np.float64).ravel()
    return float(np.sqrt(np.sum((e - a) ** 2) / max(np.sum(e * e), 1e-30)))


@pytest.fixture(scope="module")
def tiny(oracle_lib):
    from oracle.decoder import load_tiny
    return load_tiny(GOLDEN)


def test_fp32_every_layer_matches_transformers(tiny):
    """Qwen35ParityTests.EveryLayerMatchesTransformers (:45-86)."""
    from oracle.decoder import OracleDecoder
    cfg, w, ids, ref, _ = tiny
    states, last = OracleDecoder(cfg, w).forward(ids)
    checked = 0
    for name, got in states.items():
        if name not in ref:
            continue
        ours, theirs = rel(ref["fp64." + name], got), rel(ref["fp64." + name], ref[name])
        assert ours <= 2 * theirs + 1e-7, (name, ours, theirs)
        assert rel(ref[name], got) < 1e-4, (name, rel(ref[name], got))
        checked += 1
    assert checked == 2 * cfg.layers + 1
    logits = OracleDecoder(cfg, w).logits(last, list(range(cfg.vocab)))
    assert rel(ref["logits"], logits) < 1e-4
    assert rel(ref["fp64.logits"], logits) <= 2 * rel(ref["fp64.logits"], ref["logits"]) + 1e-7


def test_q8_0_matches_transformers_computing_as_ggml(tiny):
    """Qwen35ParityTests.Q8_0MatchesTransformersComputingAsGgml (:95-136)."""
    from oracle.decoder import OracleDecoder
    cfg, w, ids, ref, refq = tiny
    m = OracleDecoder(cfg, w, precision="q8_0")
    states, last = m.forward(ids)
    for name, want in refq.items():
        if name not in states:
            continue
        between, quantization = rel(want, states[name]), rel(ref[name], want)
        assert between <= 0.2 * quantization, (name, between, quantization)
        if name == "layers.0.mixer":
            assert between < 1e-4
    logits = m.logits(last, list(range(cfg.vocab)))
    assert rel(refq["logits"], logits) <= 0.2 * rel(ref["logits"], refq["logits"])


def test_delta_rule_is_the_two_sweep_recurrence(oracle_lib):
    """lo_delta_rule against a float64-free restatement of the recurrence written out per element (S·g, m = Sᵀk,
    δ = (v − m)β, S += k ⊗ δ, o = Sᵀq) on random data: identical."""
    import math
    rng = np.random.default_rng(0)
    dk, dv, T = 8, 8, 5
    q, k, v = (rng.standard_normal((T, dk)).astype(np.float32) for _ in range(3))
    v = rng.standard_normal((T, dv)).astype(np.float32)
    g = rng.uniform(0.5, 1, T).astype(np.float32)
    b = rng.uniform(0, 1, T).astype(np.float32)
    qkv = np.concatenate([q, k, v], 1).astype(np.float32)
    state = np.zeros((dk, dv), np.float32)
    out = np.zeros((T, dv), np.float32)
    flat = qkv.reshape(-1)
    oracle_lib.lib().lo_delta_rule(state, dk, dv, T, np.ascontiguousarray(flat[0:]), np.ascontiguousarray(flat[dk:]),
                                   np.ascontiguousarray(flat[2 * dk:]), 2 * dk + dv, g, b, 1, out.reshape(-1), dv)
    S = np.zeros((dk, dv), np.float32)
    for t in range(T):
        S = (S * g[t]).astype(np.float32)
        m = np.zeros(dv, np.float32)
        for i in range(dk):
            m = np.array([math.fma(float(S[i, j]), float(k[t, i]), float(m[j])) for j in range(dv)], np.float32) \
                if hasattr(math, "fma") else (m + S[i] * k[t, i]).astype(np.float32)
        d = ((v[t] - m) * b[t]).astype(np.float32)
        o = np.zeros(dv, np.float32)
        for i in range(dk):
            if hasattr(math, "fma"):
                S[i] = np.array([math.fma(float(d[j]), float(k[t, i]), float(S[i, j])) for j in range(dv)], np.float32)
                o = np.array([math.fma(float(S[i, j]), float(q[t, i]), float(o[j])) for j in range(dv)], np.float32)
            else:
                S[i] = (S[i] + d * k[t, i]).astype(np.float32)
                o = (o + S[i] * q[t, i]).astype(np.float32)
        np.testing.assert_allclose(out[t], o, rtol=0 if hasattr(math, "fma") else 1e-6, atol=0 if hasattr(math, "fma") else 1e-6)
    np.testing.assert_allclose(state, S, rtol=0 if hasattr(math, "fma") else 1e-6, atol=0 if hasattr(math, "fma") else 1e-6)


def test_reading_in_pieces_is_exactly_reading_at_once(tiny):
    """Qwen35ParityTests.ReadingInPiecesIsExactlyReadingAtOnce (:139-157), on the oracle's state."""
    from oracle.decoder import OracleDecoder
    cfg, w, ids, _, _ = tiny
    m = OracleDecoder(cfg, w, precision="q8_0")
    _, once = m.forward(ids, record=False)
    state = m.new_state()
    m.forward(ids[:61], record=False, state=state)
    branch = state.clone()
    m.forward(ids[61:101], record=False, state=state)
    _, pieces = m.forward(ids[101:], record=False, state=state)
    assert np.array_equal(once, pieces) and state.length == len(ids)
    assert branch.length == 61
    _, again = m.forward(ids[61:], record=False, state=branch)
    assert np.array_equal(once, again)


def test_rewinding_to_a_mark_reads_the_same_as_a_fresh_state(tiny):
    """Qwen35StateTests.RewindingToAMarkReadsTheSameAsAFreshState (:176-196)."""
    from oracle.decoder import OracleDecoder
    cfg, w, _, _, _ = tiny
    m = OracleDecoder(cfg, w)
    prefix = [(i * 37) % 128 for i in range(70)]
    a, b = [5, 9, 11, 100], [7, 7, 7, 7, 7, 7, 1]
    state = m.new_state()
    m.forward(prefix, record=False, state=state)
    mark = state.save()
    _, first = m.forward(a, record=False, state=state)
    state.rewind(mark)
    _, second = m.forward(b, record=False, state=state)
    assert np.array_equal(m.forward(prefix + a, record=False)[1], first)
    assert np.array_equal(m.forward(prefix + b, record=False)[1], second)
    with pytest.raises(ValueError):
        m.new_state().rewind(mark)


def test_checkpoints_are_the_states_of_shorter_reads(tiny):
    """Qwen35BatchTests.CheckpointsAreTheStatesOfShorterReads (:233-252)."""
    from oracle.decoder import OracleDecoder
    cfg, w, _, _, _ = tiny
    m = OracleDecoder(cfg, w, precision="q8_0")
    tokens = [(i * 37 + 5 * 11) % 128 for i in range(60)]
    rest = [(i * 37 + 6 * 11) % 128 for i in range(9)]
    _, _, snaps = m.forward(tokens, record=False, state=m.new_state(), checkpoints=[5, 16, 33])
    for at, snap in zip([5, 16, 33], snaps):
        assert snap.length == at
        ref = m.new_state()
        m.forward(tokens[:at], record=False, state=ref)
        assert np.array_equal(m.forward(rest, record=False, state=ref)[1], m.forward(rest, record=False, state=snap)[1])
