"""The K-split rule of the accumulating bf16 products (laya_b200/csrc/ksplit.h), compiled by the host C++ compiler.

Weight gradients dW += dYᵀ·X have few output tiles over K = tokens; their K is split into chunks whose partial tiles
reduce-add into the gradient. Checked here on CPU: the chunk counts of the config-3 weight-gradient shapes, that every
chunk is non-empty and at least 4 k-blocks long, that many output tiles are never split, and that the choice has the
smallest (rounds of units over the SMs) × (k-blocks per unit + 1) of all admissible chunk counts.
"""
import itertools
import os
import subprocess

import pytest

from conftest import ROOT

CASES = [(t, kb, nsm) for t, kb, nsm in itertools.product([1, 3, 9, 18, 27, 30, 54, 100, 147, 148, 480],
                                                         [1, 3, 4, 7, 8, 12, 36, 160, 320, 321, 1024], [132, 148])]


@pytest.fixture(scope="module")
def chosen(tmp_path_factory):
    d = tmp_path_factory.mktemp("ksplit")
    src = d / "ks.cpp"
    src.write_text('#include <cstdio>\n#include "ksplit.h"\nint main() {\n'
                   + "".join(f'    std::printf("%d\\n", laya::bf::choose_ksplit({t}, {kb}, {n}));\n' for t, kb, n in CASES)
                   + "    return 0;\n}\n")
    exe = d / "ks"
    subprocess.check_call(["g++", "-std=c++17", "-O1", "-I" + os.path.join(ROOT, "laya_b200", "csrc"), str(src), "-o", str(exe)])
    return dict(zip(CASES, (int(v) for v in subprocess.check_output([str(exe)]).split())))


def cost(tiles, kblocks, nsm, ks):
    kchunk = -(-kblocks // ks)
    return -(-tiles * ks // nsm) * (kchunk + 1)


def test_config3_weight_gradients(chosen):
    # 20480 tokens = 320 k-blocks; 128 x 256 output tiles of dW for Wqkv / Wi (2304 x 768: 54 tiles), Wo (768 x 768:
    # 18) and the MLP out (768 x 1152: 30)
    assert chosen[(54, 320, 148)] == 8      # 432 units: 3 rounds, the last nearly full (6 chunks: the last a fifth full)
    assert chosen[(18, 320, 148)] == 8      # 144 units: one round
    assert chosen[(30, 320, 148)] == 14     # 420 units: 3 rounds, the last 84% full


def test_chunks_are_admissible_and_the_cost_is_minimal(chosen):
    for (tiles, kblocks, nsm), ks in chosen.items():
        if tiles >= nsm:
            assert ks == 1                   # enough output tiles: never split
            continue
        assert ks >= 1
        kchunk = -(-kblocks // ks)
        assert (ks - 1) * kchunk < kblocks <= ks * kchunk          # every chunk non-empty
        if ks > 1:
            assert kchunk >= 4                                     # chunks of at least 4 k-blocks
        admissible = {-(-kblocks // -(-kblocks // w)) for w in range(1, max(1, kblocks // 4) + 1)}
        assert ks in admissible
        assert cost(tiles, kblocks, nsm, ks) == min(cost(tiles, kblocks, nsm, a) for a in admissible)
