"""Decoder states on the B200 (include/laya_decoder.h: laya_decoder_state_*, laya_decoder_forward_states).

Qwen35State (Mica/Models/Qwen35Model.cs:38-197) promises that reading a prompt in pieces through one state gives bit
for bit the activations of reading it at once; Mica's shared-prefix reuse (MicaJudge.cs:166-229) rests on it.  These
are the reference's own state tests (Qwen35ParityTests.cs:139-157, Qwen35StateTests :176-196, Qwen35BatchTests
:209-252) on the device path, bit-exact against the device's own one-pass read — whose parity with the oracle and the
qwen35-tiny fixture is test_decoder_gpu.py's — plus the fixture's own bar for a read in pieces, cache growth past the
decoder's first RoPE table, and the rejected calls that must leave a state untouched.
"""
import numpy as np
import pytest

from conftest import GOLDEN
from test_decoder_gpu import desc_of, rel

pytestmark = pytest.mark.gpu


def tokens(count, seed):
    """Qwen35BatchTests.Tokens (Qwen35ParityTests.cs:207)."""
    return np.array([(i * 37 + seed * 11) % 128 for i in range(count)], np.int64)


@pytest.fixture(scope="module")
def model(cuda):
    import laya_b200
    from oracle.decoder import load_tiny
    cfg, w, ids, ref, refq = load_tiny(GOLDEN)
    m = laya_b200.Qwen35Model(desc_of(cfg, max_tokens=512, max_seqs=8), device=0)
    m.load(w)
    yield cfg, w, ids, ref, refq, m
    m.close()


def once(m, seq, labels=None):
    h, lg = m.forward([seq], labels)
    return h[0] if labels is None else (h[0], lg[0])


def test_reading_in_pieces_is_exactly_reading_at_once(model):
    """ReadingInPiecesIsExactlyReadingAtOnce (:139-157)."""
    cfg, _, ids, ref, refq, m = model
    whole = once(m, ids)
    state = m.new_state()
    m.forward_state(ids[:61], state)
    branch = state.clone()
    m.forward_state(ids[61:101], state)
    pieces = m.forward_state(ids[101:], state)
    assert np.array_equal(whole.view(np.uint32), pieces.view(np.uint32))
    assert state.length == len(ids)
    assert branch.length == 61
    assert np.array_equal(whole.view(np.uint32), m.forward_state(ids[61:], branch).view(np.uint32))
    # the fixture's bar (Qwen35ParityTests.cs:95-136) holds for the read in pieces
    logits = m.logits(pieces, list(range(cfg.vocab)))[0]
    assert rel(refq["logits"], logits) <= 0.2 * rel(ref["logits"], refq["logits"])
    assert state.bytes > 0
    for s in (state, branch):
        s.close()


def test_rewinding_to_a_mark_reads_the_same_as_a_fresh_state(model):
    """Qwen35StateTests.RewindingToAMarkReadsTheSameAsAFreshState (:176-196)."""
    import laya_b200
    _, _, _, _, _, m = model
    prefix = np.array([(i * 37) % 128 for i in range(70)], np.int64)
    a, b = np.array([5, 9, 11, 100]), np.array([7, 7, 7, 7, 7, 7, 1])
    state = m.new_state(16)
    m.forward_state(prefix, state)
    mark = state.save()
    first = m.forward_state(a, state)
    state.rewind(mark)
    assert state.length == 70
    second = m.forward_state(b, state)
    assert np.array_equal(once(m, np.concatenate([prefix, a])).view(np.uint32), first.view(np.uint32))
    assert np.array_equal(once(m, np.concatenate([prefix, b])).view(np.uint32), second.view(np.uint32))
    fresh = m.new_state()
    with pytest.raises(laya_b200.LayaArgumentError):
        fresh.rewind(mark)   # a mark can only rewind
    for x in (mark, state, fresh):
        x.close()


def test_a_batch_reads_each_sequence_exactly_as_alone(model):
    """Qwen35BatchTests.ABatchReadsEachSequenceExactlyAsAlone (:209-230), with label logits."""
    import laya_b200
    _, _, _, _, _, m = model
    prefix = tokens(50, 1)
    suffixes = [tokens(7, 2), tokens(1, 3), tokens(30, 4), tokens(70, 7)]
    labels = [3, 17, 99]
    expected = [once(m, np.concatenate([prefix, s]), labels) for s in suffixes]
    shared = m.new_state()
    m.read(prefix, shared)
    branches = [laya_b200.Qwen35Sequence(s, shared.clone()) for s in suffixes]
    m.forward_sequences(branches, labels)
    for (h, lg), q, s in zip(expected, branches, suffixes):
        assert np.array_equal(h.view(np.uint32), q.hidden.view(np.uint32))
        assert np.array_equal(lg.view(np.uint32), q.logits.view(np.uint32))
        assert q.state.length == len(prefix) + len(s)
    assert shared.length == len(prefix)
    for q in branches:
        q.state.close()
    shared.close()


def test_checkpoints_are_the_states_of_shorter_reads(model):
    """Qwen35BatchTests.CheckpointsAreTheStatesOfShorterReads (:233-252), a checkpoint at the read's end included,
    two sequences with checkpoints in one pass."""
    import laya_b200
    _, _, _, _, _, m = model
    toks, rest = tokens(60, 5), tokens(9, 6)
    other = tokens(45, 8)
    seqs = [laya_b200.Qwen35Sequence(toks, m.new_state(), readout=False, checkpoints=[5, 16, 33, 60]),
            laya_b200.Qwen35Sequence(other, m.new_state(), readout=True, checkpoints=[1, 44])]
    m.forward_sequences(seqs)
    for q in seqs:
        assert len(q.snapshots) == len(q.checkpoints)
        for at, snap in zip(q.checkpoints, q.snapshots):
            assert snap.length == at
            ref = m.new_state()
            m.read(q.tokens[:at], ref)
            want = m.forward_state(rest, ref)
            assert np.array_equal(want.view(np.uint32), m.forward_state(rest, snap).view(np.uint32)), at
            ref.close()
            snap.close()
        q.state.close()


def test_a_state_grows_past_the_first_rope_table(model, cuda):
    """Keys and values grow on demand (Qwen35State.GrowCache, :146-154) and positions past the decoder's max_tokens
    get their RoPE rows: 1200 tokens read in three pieces on a decoder of 512-token forwards equal one 1200-token
    forward of a decoder sized for it."""
    import laya_b200
    cfg, w, _, _, _, m = model
    seq = tokens(1200, 9)
    big = laya_b200.Qwen35Model(desc_of(cfg, max_tokens=1280, max_seqs=2), device=0)
    big.load(w)
    whole = once(big, seq)
    state = m.new_state(100)
    m.read(seq[:500], state)
    m.read(seq[500:900], state)
    last = m.forward_state(seq[900:], state)
    assert np.array_equal(whole.view(np.uint32), last.view(np.uint32))
    assert state.length == 1200
    state.close()
    big.close()


def test_rejected_calls_leave_the_state_as_it_was(model):
    import laya_b200
    cfg, _, _, _, _, m = model
    prefix, more = tokens(30, 10), tokens(12, 11)
    s = m.new_state()
    m.read(prefix, s)
    bad = more.copy()
    bad[5] = cfg.vocab
    with pytest.raises(laya_b200.LayaOutOfRangeError):
        m.forward_state(bad, s)
    with pytest.raises(laya_b200.LayaArgumentError):   # the same state twice in one pass
        m.forward_sequences([laya_b200.Qwen35Sequence(more, s), laya_b200.Qwen35Sequence(more, s)])
    with pytest.raises(laya_b200.LayaArgumentError):   # checkpoints must ascend within the read
        m.forward_sequences([laya_b200.Qwen35Sequence(more, s, checkpoints=[4, 4])])
    with pytest.raises(laya_b200.LayaArgumentError):
        m.forward_sequences([laya_b200.Qwen35Sequence(more, s, checkpoints=[13])])
    assert s.length == 30
    assert np.array_equal(once(m, np.concatenate([prefix, more])).view(np.uint32),
                          m.forward_state(more, s).view(np.uint32))
    s.close()
