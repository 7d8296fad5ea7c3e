"""The data-parallel fine-tuning step on 2 B200s: NCCL-bucketed gradient sums inside the library.

Two ranks each train half of the training-tiny batch and take one clipped AdamW step; the result must equal (to fp32
summation order) one GPU accumulating both halves at scale 1/2 and stepping once, and be bit-identical across the
ranks.  Skipped on a machine with fewer than two GPUs.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_two_ranks_equal_one_gpu_accumulating(cuda, tmp_path):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "dp_worker.py"), str(tmp_path)]
    r = subprocess.run(cmd, capture_output=True, text=True, env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    r0, r1, single = (dict(np.load(tmp_path / f)) for f in ("rank0.npz", "rank1.npz", "single.npz"))
    assert float(r0["norm"]) == float(r1["norm"])
    assert abs(float(r0["norm"]) - float(single["norm"])) <= 1e-5 * float(single["norm"])
    for k in single:
        if k == "norm":
            continue
        assert np.array_equal(r0[k], r1[k]), k
        assert np.allclose(r0[k], single[k], rtol=0, atol=2e-7), (k, np.abs(r0[k] - single[k]).max())
