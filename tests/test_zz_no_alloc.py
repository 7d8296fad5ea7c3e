"""laya_q8_0_linear_noalloc: the Q8_0 projection for callers that cannot allocate device memory.

Those callers (hosts whose device memory belongs to their own pool under a fixed budget, plugins that may not grow
another process's footprint) hand in every buffer themselves; the entry point's only scratch is a static device
array inside the library.  This checks it against the allocating path — activation quantizer + product on caller
buffers — on two calls in a row, which also exercises the shared scratch keeping the previous call's contents.
Collected last so that a failure here never hides the other tests of a run that stops at the first failure.
"""
import ctypes

import numpy as np
import pytest

from conftest import bits

pytestmark = pytest.mark.gpu


def _weight(torch, laya_b200, ctx, rng, N, K):
    w = torch.from_numpy(rng.normal(0, 0.05, (N, K)).astype(np.float32)).cuda()
    ldw = (N + 127) // 128 * 128
    codes = torch.zeros((N, K), dtype=torch.float16, device="cuda")
    scales = torch.zeros((K // 32, ldw), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.quantize_weights(ctx, w.data_ptr(), N, K, codes.data_ptr(), scales.data_ptr(), ldw)
    return codes, scales, ldw


def _allocating_path(torch, laya_b200, ctx, x, rows, stride, codes, scales, ldw, N, K, bias):
    ldx = (rows + 127) // 128 * 128
    qx = torch.zeros((rows, K), dtype=torch.float16, device="cuda")
    dx = torch.zeros((K // 32, ldx), dtype=torch.float32, device="cuda")
    y = torch.zeros((rows, N), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.quantize_activations(ctx, x.data_ptr(), rows, stride, K, qx.data_ptr(), dx.data_ptr(), ldx)
    laya_b200.Q8_0.gemm(ctx, qx.data_ptr(), dx.data_ptr(), ldx, rows, codes.data_ptr(), scales.data_ptr(), ldw, N, K,
                        bias.data_ptr() if bias is not None else None, y.data_ptr(), N)
    return y


def test_no_alloc_projection_equals_the_allocating_one(cuda):
    torch = cuda
    import laya_b200
    L = laya_b200.lib()
    ctx = laya_b200.Context(laya_b200.base_desc(max_tokens=256, max_items=4, max_markers=16))
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(17)
    N, K = 768, 1152
    codes, scales, ldw = _weight(torch, laya_b200, ctx, rng, N, K)
    bias = torch.from_numpy(rng.normal(size=N).astype(np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (rows, stride) in enumerate([(1000, K + 3), (317, K)]):
        x = torch.from_numpy(rng.normal(0, 1, (rows, stride)).astype(np.float32)).cuda()
        y = torch.full((rows, N), float("nan"), dtype=torch.float32, device="cuda")
        laya_b200.api.check(L.laya_q8_0_linear_noalloc(
            x.data_ptr(), rows, stride, codes.data_ptr(), scales.data_ptr(), ldw, N, K, bias.data_ptr(), y.data_ptr(),
            N, stream))
        want = _allocating_path(torch, laya_b200, ctx, x, rows, stride, codes, scales, ldw, N, K, bias)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y.cpu().numpy()), bits(want.cpu().numpy())), f"call {call} differs"
    ctx.close()


def _need(rows, K):
    """Bytes of the static scratch one call takes: a 256-byte status word, the codes [rows, K] (2 bytes each, padded
    to 256 bytes) and the block scales [K/32, rows rounded up to 128] (4 bytes each)."""
    ldx = (rows + 127) // 128 * 128
    return 256 + (rows * K * 2 + 255) // 256 * 256 + (K // 32) * ldx * 4


def _largest_rows(K, limit=8 << 20):
    rows = limit // (2 * K)
    while _need(rows, K) > limit:
        rows -= 1
    return rows


@pytest.mark.parametrize("K", [3072, 9216])
def test_no_alloc_at_the_scratch_limit(cuda, K):
    """The largest call that fits the scratch equals the allocating path bit for bit, twice (the second call with
    fewer rows, so it reads scales the first call left in the padded rows), and one row more is rejected."""
    torch = cuda
    import laya_b200
    L = laya_b200.lib()
    rows = _largest_rows(K)
    assert _need(rows, K) <= 8 << 20 < _need(rows + 1, K)
    ctx = laya_b200.Context(laya_b200.base_desc(max_tokens=256, max_items=4, max_markers=16))
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(K)
    N = 256
    codes, scales, ldw = _weight(torch, laya_b200, ctx, rng, N, K)
    stream = torch.cuda.current_stream().cuda_stream
    for call, r in enumerate([rows, rows - 77]):
        x = torch.from_numpy(rng.normal(0, 1, (r, K)).astype(np.float32)).cuda()
        y = torch.full((r, N), float("nan"), dtype=torch.float32, device="cuda")
        laya_b200.api.check(L.laya_q8_0_linear_noalloc(
            x.data_ptr(), r, K, codes.data_ptr(), scales.data_ptr(), ldw, N, K, None, y.data_ptr(), N, stream))
        want = _allocating_path(torch, laya_b200, ctx, x, r, K, codes, scales, ldw, N, K, None)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y.cpu().numpy()), bits(want.cpu().numpy())), f"K={K} call {call} differs"
    x = torch.zeros((rows + 1, K), dtype=torch.float32, device="cuda")
    y = torch.zeros((rows + 1, N), dtype=torch.float32, device="cuda")
    rc = L.laya_q8_0_linear_noalloc(x.data_ptr(), rows + 1, K, codes.data_ptr(), scales.data_ptr(), ldw, N, K, None,
                                    y.data_ptr(), N, stream)
    assert rc == 1 and b"scratch" in L.laya_last_error()
    ctx.close()


def test_no_alloc_rejects_calls_beyond_its_scratch(cuda):
    torch = cuda
    import laya_b200
    L = laya_b200.lib()
    scratch = 8 << 20
    K, N = 3072, 64
    rows = scratch // (2 * K) + 128          # codes alone exceed the scratch
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    rc = L.laya_q8_0_linear_noalloc(dummy.data_ptr(), rows, K, dummy.data_ptr(), dummy.data_ptr(), 64, N, K, None,
                                    dummy.data_ptr(), N, None)
    assert rc == 1 and b"scratch" in L.laya_last_error()
    rc = L.laya_q8_0_linear_noalloc(dummy.data_ptr(), 4, 40, dummy.data_ptr(), dummy.data_ptr(), 64, N, 40, None,
                                    dummy.data_ptr(), N, None)
    assert rc == 1
