"""The AVX-512 restatements of the reference's panel kernels (oracle/laya_vnni.c) that time the CPU baseline give the
same bits as the scalar definitions the parity tests use (skipped on a CPU without AVX-512 VNNI)."""
import numpy as np
import pytest

import oracle


@pytest.fixture(scope="module")
def fast():
    oracle.build()
    if oracle.vnni_lib() is None:
        pytest.skip("this CPU has no AVX-512 VNNI")
    yield
    oracle.set_fast(False)


@pytest.mark.parametrize("rows,N,K", [(1, 64, 32), (5, 100, 96), (37, 2304, 768), (3, 768, 1152)])
def test_q8_panel_kernel_equals_the_definition(fast, rows, N, K):
    """PackedMatrixQ8_0.Panel512's vpdpbusd form (unsigned-offset activations, −128·Σw start) against the per-block
    definition: exact block sums, then fma((float)Σ, d_w·d_x, acc) in block order — bit for bit, with and without
    bias, N not a multiple of the 64-column panel, rows not a multiple of three."""
    rng = np.random.default_rng(rows * 7 + N)
    x = rng.normal(0, 1, (rows, K)).astype(np.float32)
    w = rng.normal(0, 0.05, (N, K)).astype(np.float32)
    qw, dw = oracle.q8_quantize_weights(w)
    qx, dx = oracle.q8_quantize_activations(x)
    bias = rng.normal(size=N).astype(np.float32)
    for b in (None, bias):
        oracle.set_fast(False)
        want = oracle.q8_matmul(qx, dx, qw, dw, b)
        oracle.set_fast(True)
        got = oracle.q8_matmul(qx, dx, qw, dw, b)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,N,K", [(1, 64, 16), (6, 130, 77), (9, 1024, 1024)])
def test_f32_panel_kernel_equals_the_definition(fast, rows, N, K):
    """PackedMatrix.Multiply's panel form against acc = bias, then one fma per input feature in increasing order."""
    rng = np.random.default_rng(rows + N + K)
    x = rng.normal(0, 1, (rows, K)).astype(np.float32)
    w = rng.normal(0, 0.05, (N, K)).astype(np.float32)
    bias = rng.normal(size=N).astype(np.float32)
    for b in (None, bias):
        oracle.set_fast(False)
        want = oracle.linear_f32(x, w, b)
        oracle.set_fast(True)
        got = oracle.linear_f32(x, w, b)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("window,rope", [(-1, True), (64, True), (7, False)])
def test_attention_kernel_equals_the_restatement(fast, window, rope):
    """AttentionKernels' key-transposed scores and dimension-vectorised weighted sum against lo_attention, bit for
    bit: ragged segments (one shorter than a 16-key vector, one past the window), global and sliding, with and
    without rotary."""
    rng = np.random.default_rng(window + 100)
    hidden, heads = 256, 4
    seg_len = np.array([5, 150, 71], np.int32)
    seg_start = np.concatenate([[0], np.cumsum(seg_len)[:-1]]).astype(np.int32)
    qkv = rng.normal(0, 1, (int(seg_len.sum()), 3 * hidden)).astype(np.float32)
    tables = oracle.rope_table(hidden // heads, 10000.0, int(seg_len.max())) if rope else None
    oracle.set_fast(False)
    want = oracle.attention(qkv, hidden, heads, seg_start, seg_len, window, tables)
    oracle.set_fast(True)
    got = oracle.attention(qkv, hidden, heads, seg_start, seg_len, window, tables)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
