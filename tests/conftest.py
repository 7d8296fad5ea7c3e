"""Shared test setup: repository root on sys.path, the `gpu` marker, and helpers."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built liblaya_b200.so")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    """The GPU tests run only on a B200 box; there they must find the library (no fallback)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a machine without CUDA")
    import laya_b200
    laya_b200.lib()          # raises LayaLibraryMissing when the build is absent
    return torch


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def max_rel(a, b):
    """max |a - b| / max |b| — the scale-relative error the parity bars are stated in."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))
