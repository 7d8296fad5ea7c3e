"""Data-parallel semantics of the fine-tuning step on CPU ranks (gloo, world size 2).

The device trainer sums gradients over the ranks (NCCL, 25 MB buckets) and applies clip + AdamW to their average:
clip coefficient max_norm / (||Σg|| / world + 1e-6), factor min(1, coef) / world on the summed gradient.  Checked
here on the oracle: two ranks with one half of the batch each, gloo allreduce, that rule — against one process that
accumulates both halves at scale 1/2 (the RLCD objective's 1/accumulation scale) and steps once.  Also the exchange
of the 128-byte NCCL id that bench.py and the trainer use.
"""
import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import GOLDEN

MAX_NORM = 0.05


def _tiny():
    from oracle.model import EncoderConfig
    g = json.load(open(os.path.join(GOLDEN, "training_tiny.json")))
    w = dict(np.load(os.path.join(GOLDEN, "training_tiny_model.npz")))
    cfg = EncoderConfig.from_hf(g["encoder_config"], head_layers=2, n_act=2)
    return cfg, w, g["batch"]["items"]


def _grads(cfg, w, items, scale):
    from oracle.train import TorchTrainModel
    m = TorchTrainModel(cfg, w)
    logits = m.forward(items)
    sum((l * torch.tensor(it["coeff"]) * scale).sum() for l, it in zip(logits, items)).backward()
    return {k: v.astype(np.float64) for k, v in m.grads().items()}


def _step(w, grads, coef_factor):
    from oracle.train import adamw_step
    out = {}
    for k, v in w.items():
        if k == "temperature":
            continue
        p = v.astype(np.float32).reshape(-1).copy()
        m_ = np.zeros_like(p)
        v_ = np.zeros_like(p)
        adamw_step(p, (grads[k].reshape(-1) * coef_factor).astype(np.float32), m_, v_, 1, 1e-4)
        out[k] = p
    return out


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg, w, items = _tiny()
    mine = items[:2] if rank == 0 else items[2:]
    g = _grads(cfg, w, mine, 1.0)
    names = sorted(g)
    flat = torch.from_numpy(np.concatenate([g[k].ravel() for k in names]))
    dist.all_reduce(flat, op=dist.ReduceOp.SUM)                  # the bucketed NCCL sum, in one piece
    summed, o = {}, 0
    for k in names:
        summed[k] = flat[o:o + g[k].size].numpy().reshape(g[k].shape)
        o += g[k].size
    norm = float(np.sqrt(sum(np.sum(v ** 2) for v in summed.values()))) / world
    coef = MAX_NORM / (norm + 1e-6)
    factor = min(1.0, coef) / world
    params = _step(w, summed, factor)
    uid = [os.urandom(128) if rank == 0 else None]               # the NCCL id exchange of bench.py
    dist.broadcast_object_list(uid, src=0)
    gathered = [None] * world
    dist.all_gather_object(gathered, uid[0])
    q.put((rank, norm, {k: v for k, v in params.items()}, gathered[0] == gathered[1] and len(uid[0]) == 128))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_average_like_accumulation():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort(key=lambda r: r[0])
    (_, n0, p0, ok0), (_, n1, p1, ok1) = res
    assert ok0 and ok1
    assert n0 == n1
    for k in p0:
        assert np.array_equal(p0[k], p1[k]), k                  # every rank applies the same update
    # one process, both halves accumulated at scale 1/2, one clipped step
    cfg, w, items = _tiny()
    g = {k: a + b for (k, a), b in zip(_grads(cfg, w, items[:2], 0.5).items(), _grads(cfg, w, items[2:], 0.5).values())}
    norm = float(np.sqrt(sum(np.sum(v ** 2) for v in g.values())))
    assert abs(norm - n0) <= 1e-6 * norm
    ref = _step(w, g, min(1.0, MAX_NORM / (norm + 1e-6)))
    for k in ref:
        assert np.allclose(p0[k], ref[k], rtol=0, atol=1e-7), k
