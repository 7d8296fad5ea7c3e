"""Checkpoint I/O on the device trainer (include/laya_train.h: laya_trainer_save_checkpoint / _restore_checkpoint).

TrainableDecisionModel.Save (TrainableDecisionModel.cs:649-661) writes model.safetensors through SafetensorsWriter
(Base/Io/SafetensorsWriter.cs:17-64): every parameter in the dtype it was read in, bf16 by round-to-nearest-even.
Checked here: the file's layout and bytes as that writer would produce them, a restore that reproduces every
parameter bit for bit, and — with AdamW's state, which the reference does not save — a resumed run that continues
the uninterrupted one bit for bit.
"""
import json
import os
import struct

import numpy as np
import pytest

from test_train_gpu import desc_for, fixture_items, tiny

pytestmark = pytest.mark.gpu


def read_safetensors(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    return header, data


def to_bf16_bits(x):
    """SafetensorsWriter.ToBFloat16: round to nearest even on the top 16 bits."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def make(cfg, w, bf16_names=()):
    import laya_b200
    t = laya_b200.Trainer(desc_for(cfg, max_tokens=256, max_items=16, max_markers=64),
                          laya_b200.train_desc(max_segment=128), device=0)
    for name, arr in w.items():
        if name == "temperature":
            continue
        if name in bf16_names:
            t.upload(name, to_bf16_bits(arr), dtype=laya_b200.api.BF16)
        else:
            t.upload(name, arr)
    return t


def step(t, g, b):
    items = g["batch"]["items"]
    t.zero_grads()
    t.forward(b, training=False)
    t.backward(b, [np.array(it["coeff"], np.float32) * 50 for it in items])
    t.clip_and_step(max_norm=0.5)


def test_save_restore_and_resume(cuda, tmp_path):
    cfg, w, g = tiny()
    bf16 = ("encoder.embeddings.tok_embeddings.weight", "head.layers.0.linear1.weight")
    a = make(cfg, w, bf16)
    a.set_lr(2.5e-5, 1e-4)
    ba = a.batch(fixture_items(g))
    step(a, g, ba)
    path = str(tmp_path / "model.safetensors")
    a.save_checkpoint(path, with_optimizer=True)
    names = a.names()

    # the file: SafetensorsWriter's layout, dtypes as uploaded, payloads as that writer rounds them
    header, data = read_safetensors(path)
    assert header["__metadata__"]["optimizer_step"] == "1"
    for n, r, c in names:
        e = header[n]
        got_shape = [int(x) for x in e["shape"]]
        assert got_shape == (list(w[n].shape) if n in w else got_shape), n
        lo, hi = e["data_offsets"]
        master = a.download(n, (r, c)).ravel()
        if n in bf16:
            assert e["dtype"] == "BF16"
            assert np.array_equal(np.frombuffer(data[lo:hi], np.uint16), to_bf16_bits(master)), n
        else:
            assert e["dtype"] == "F32"
            assert np.array_equal(np.frombuffer(data[lo:hi], np.uint32), master.view(np.uint32)), n
        assert f"optimizer.m.{n}" in header and f"optimizer.v.{n}" in header

    # restore into a fresh trainer: every parameter bit for bit (the bf16-stored ones as their rounded values)
    b = make(cfg, {k: np.zeros_like(v) for k, v in w.items()})
    b.restore_checkpoint(path)
    assert b.steps() == 1
    for n, r, c in names:
        want = a.download(n, (r, c)).ravel()
        if n in bf16:
            want = (to_bf16_bits(want).astype(np.uint32) << 16).view(np.float32)
        assert np.array_equal(b.download(n, (r, c)).ravel().view(np.uint32), want.view(np.uint32)), n

    # resume: with the optimizer state, a step on the restored trainer equals the same step on a trainer restored
    # from a save without rounding (all F32) — and one without the state is a different trajectory
    a32 = make(cfg, w)
    a32.set_lr(2.5e-5, 1e-4)
    b32a = a32.batch(fixture_items(g))
    step(a32, g, b32a)
    p32 = str(tmp_path / "f32.safetensors")
    a32.save_checkpoint(p32, with_optimizer=True)
    c = make(cfg, {k: np.zeros_like(v) for k, v in w.items()})
    c.restore_checkpoint(p32)
    c.set_lr(2.5e-5, 1e-4)
    bc = c.batch(fixture_items(g))
    step(a32, g, b32a)
    step(c, g, bc)
    assert c.steps() == a32.steps() == 2
    for n, r, cc in names:
        assert np.array_equal(c.download(n, (r, cc)).ravel().view(np.uint32),
                              a32.download(n, (r, cc)).ravel().view(np.uint32)), n
    p_noopt = str(tmp_path / "noopt.safetensors")
    a32.save_checkpoint(p_noopt, with_optimizer=False)
    h2, _ = read_safetensors(p_noopt)
    assert "__metadata__" not in h2 and not any(k.startswith("optimizer.") for k in h2)
    d = make(cfg, {k: np.zeros_like(v) for k, v in w.items()})
    d.restore_checkpoint(p_noopt)
    assert d.steps() == 0
    for x in (ba, b32a, bc):
        x.close()
    for x in (a, b, a32, c, d):
        x.close()


def test_restore_errors(cuda, tmp_path):
    import laya_b200
    cfg, w, g = tiny()
    t = make(cfg, w)
    with pytest.raises(laya_b200.LayaNotFoundError):
        t.restore_checkpoint(str(tmp_path / "missing.safetensors"))
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(struct.pack("<Q", 8) + b"not json")
    with pytest.raises(laya_b200.LayaArgumentError):
        t.restore_checkpoint(str(bad))
    # a file without one of the parameters
    t.save_checkpoint(str(tmp_path / "full.safetensors"), with_optimizer=False)
    header, data = read_safetensors(str(tmp_path / "full.safetensors"))
    drop = "scorer.3.bias"
    lo, hi = header.pop(drop)["data_offsets"]
    js = json.dumps(header).encode()
    js += b" " * (-len(js) % 8)
    (tmp_path / "partial.safetensors").write_bytes(struct.pack("<Q", len(js)) + js + data)
    with pytest.raises(laya_b200.LayaNotFoundError):
        t.restore_checkpoint(str(tmp_path / "partial.safetensors"))
    t.close()


def test_calibrate_is_the_fit_of_the_device_logits(cuda):
    """Trainer.Calibrate (Laya.Training/Trainer.cs:200-211) on the device: forward-only passes over batches of 16,
    then TemperatureFitting.Fit — equal, bit for bit, to the oracle's fit of the same batches' logits and targets."""
    import laya_b200
    from laya_b200 import workloads
    from oracle.train import fit_temperatures
    cfg, w, g = tiny()
    t = make(cfg, w)
    batches, samples = [], []
    for i in range(3):
        items, _ = workloads.training_batch(rows=16, min_len=8, max_len=15, vocab=cfg.vocab, seed=60 + i)
        b = t.batch(items)
        batches.append(b)
        for it, z in zip(items, t.forward(b, training=False)):
            samples.append((it.question_type, z, it.target))
    got = t.calibrate(batches, minimum_bucket_samples=5)
    want = fit_temperatures(samples, 5)
    assert [np.float32(v) for v in got[0]] == [np.float32(v) for v in want[0]]
    assert {k: np.float32(v) for k, v in got[1].items()} == {k: np.float32(v) for k, v in want[1].items()}
    assert got[2] == want[2] and sum(got[2].values()) == 48
    for b in batches:
        b.close()
    t.close()
