"""Q8_0 kernels on the B200 against the oracle, through the C ABI (bit-exact: codes, scales and fp32 products).

Restates PackedMatrixQ8_0Tests (tests/StructuredDecisions.Tests/PackedMatrixQ8_0Tests.cs) for the tensor-core path.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN, bits, max_rel

pytestmark = pytest.mark.gpu

# PackedMatrixQ8_0Tests.Shapes (PackedMatrixQ8_0Tests.cs:46-55): rows, out, in, bias
SHAPES = [(1, 64, 32, False), (2, 64, 64, True), (3, 128, 96, False), (7, 130, 160, True), (13, 192, 2560, False),
          (32, 100, 288, True), (219, 256, 9216, False)]


def codes(t):
    """Device codes (fp16-held integers) as int8, checking they are integers in -127..127."""
    v = t.float().cpu().numpy()
    assert np.all(v == np.round(v)) and np.all(np.abs(v) <= 127)
    return v.astype(np.int8)


@pytest.fixture(scope="module")
def ctx(cuda):
    import laya_b200
    c = laya_b200.Context(laya_b200.base_desc(max_tokens=4096, max_items=8, max_markers=64))
    c.set_stream(cuda.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def reference_case(rows, N, K, with_bias):
    """Weights and inputs as EveryKernelIsExactlyTheDefinition builds them (PackedMatrixQ8_0Tests.cs:64-73)."""
    rng = np.random.default_rng(rows * 131 + N * 7 + K)
    w = (rng.random(N * K) * 2 - 1)
    w[::97] *= 8
    w = w.astype(np.float32).reshape(N, K)
    istride, ostride = K + 5, N + 3
    x = (rng.random(rows * istride) * 2 - 1).astype(np.float32)
    bias = rng.random(N).astype(np.float32) if with_bias else None
    return w, x, bias, istride, ostride


@pytest.mark.parametrize("rows,N,K,with_bias", SHAPES)
def test_every_shape_is_exactly_the_definition(ctx, oracle_lib, rows, N, K, with_bias):
    """PackedMatrixQ8_0Tests.EveryKernelIsExactlyTheDefinition (:57-99): same bits as the definition, strided input,
    NaN-guarded output padding untouched."""
    import laya_b200
    o = oracle_lib
    w, x, bias, istride, ostride = reference_case(rows, N, K, with_bias)
    m = laya_b200.PackedMatrixQ8_0(ctx, f"shape.{rows}.{N}.{K}", weight=w)
    out = np.full(rows * ostride, np.nan, np.float32)
    m.multiply(x, rows, istride, bias, out, ostride)
    qw, dw = o.q8_quantize_weights(w)
    qx, dx = o.q8_quantize_activations(x.reshape(rows, istride), features=K)
    want = o.q8_matmul(qx, dx, qw, dw, bias)
    got = out.reshape(rows, ostride)
    assert np.array_equal(bits(got[:, :N]), bits(want))
    assert np.all(np.isnan(got[:-1, N:])), "wrote past the row"


def test_one_matmul_matches_torch_as_ggml(ctx):
    """Qwen35ParityTests (Qwen35ParityTests.cs:118-125): bf16 weights packed on the device, within 1e-6 of torch."""
    import laya_b200
    f = np.load(os.path.join(GOLDEN, "q8_matmul.npz"))
    wbits = (f["w"].view(np.uint32) >> 16).astype(np.uint16)
    m = laya_b200.PackedMatrixQ8_0(ctx, "golden.matmul", weight=wbits)
    y = m.multiply(f["x"], 7).reshape(7, 96)
    assert np.linalg.norm(y - f["y"]) / np.linalg.norm(f["y"]) < 1e-6


def test_dequantize_gives_q_times_d(ctx, oracle_lib):
    """PackedMatrixQ8_0.Dequantize (PackedMatrixQ8_0.cs:209-218) from the device-packed weight."""
    import laya_b200
    rng = np.random.default_rng(5)
    w = (rng.random((70, 64)) * 2 - 1).astype(np.float32)
    m = laya_b200.PackedMatrixQ8_0(ctx, "deq", weight=w)
    q, d = oracle_lib.q8_quantize_weights(w)
    assert np.array_equal(m.dequantize(), q.astype(np.float32) * np.repeat(d, 32, axis=1))


def test_activation_quantizer_bits(ctx, oracle_lib, cuda):
    """Q8_0.QuantizeActivations on the device: codes and fp16 scales bit for bit, half steps included."""
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(9)
    rows, K = 300, 768
    x = (rng.normal(size=(rows, K)) * rng.choice([1e-3, 1.0, 50.0], size=(rows, 1))).astype(np.float32)
    x[0, :32] = 0
    x[0, :6] = [127, 2.5, -2.5, 3.5, -0.5, 126.49]
    x[1, :64] = np.arange(64) / 127 * 2.5          # exact half steps (tools/dump_mica_reference.py:184)
    x[2] = 0
    xt = torch.from_numpy(x).cuda()
    q = torch.zeros((rows, K), dtype=torch.float16, device="cuda")
    d = torch.zeros((K // 32, rows), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.quantize_activations(ctx, xt.data_ptr(), rows, K, K, q.data_ptr(), d.data_ptr(), rows)
    torch.cuda.synchronize()
    wq, wd = oracle_lib.q8_quantize_activations(x)
    assert np.array_equal(codes(q), wq)
    assert np.array_equal(bits(d.cpu().numpy().T), bits(wd))
    assert list(codes(q)[0, :6]) == [127, 2, -2, 4, 0, 126]


def test_weight_quantizer_bits(ctx, oracle_lib, cuda):
    """Q8_0.QuantizeWeightBlock on the device (round half away, d fp16): bit for bit."""
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(10)
    N, K = 257, 320
    w = (rng.normal(size=(N, K)) * 0.05).astype(np.float32)
    w[0, :6] = [127, 2.5, -2.5, 3.5, -0.5, 126.49]
    w[0, 6:32] = 0
    wt = torch.from_numpy(w).cuda()
    q = torch.zeros((N, K), dtype=torch.float16, device="cuda")
    d = torch.zeros((K // 32, N), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.quantize_weights(ctx, wt.data_ptr(), N, K, q.data_ptr(), d.data_ptr(), N)
    torch.cuda.synchronize()
    oq, od = oracle_lib.q8_quantize_weights(w)
    assert np.array_equal(codes(q), oq)
    assert np.array_equal(bits(d.cpu().numpy().T), bits(od))
    assert list(codes(q)[0, :6]) == [127, 3, -3, 4, -1, 126]


def _device_operands(torch, rng, M, N, K, scale=0.002):
    qx = rng.integers(-127, 128, (M, K), dtype=np.int8)
    qw = rng.integers(-127, 128, (N, K), dtype=np.int8)
    dx = np.abs(rng.normal(0, 0.05, (M, K // 32))).astype(np.float16).astype(np.float32)
    dw = np.abs(rng.normal(0, scale, (N, K // 32))).astype(np.float16).astype(np.float32)
    ldx = (M + 127) // 128 * 128
    ldw = (N + 127) // 128 * 128
    dxt = np.zeros((K // 32, ldx), np.float32)
    dxt[:, :M] = dx.T
    dwt = np.zeros((K // 32, ldw), np.float32)
    dwt[:, :N] = dw.T
    dev = dict(qx=torch.from_numpy(qx.astype(np.float16)).cuda(), qw=torch.from_numpy(qw.astype(np.float16)).cuda(),
               dx=torch.from_numpy(dxt).cuda(), dw=torch.from_numpy(dwt).cuda())
    return qx, qw, dx, dw, ldx, ldw, dev


@pytest.mark.parametrize("M,N,K", [(1000, 2304, 768), (517, 768, 3072), (4096, 768, 1152), (129, 3072, 768)])
def test_gemm_at_model_shapes_is_bit_exact(ctx, oracle_lib, cuda, M, N, K):
    """The product at the encoder's shapes (Wqkv, linear2, MLP Wo, linear1) with ragged row tiles: every fp32 output
    equals the definition, so every int32 block dot is exact."""
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(M + N + K)
    qx, qw, dx, dw, ldx, ldw, dev = _device_operands(torch, rng, M, N, K)
    bias = rng.normal(size=N).astype(np.float32)
    bt = torch.from_numpy(bias).cuda()
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.gemm(ctx, dev["qx"].data_ptr(), dev["dx"].data_ptr(), ldx, M, dev["qw"].data_ptr(),
                        dev["dw"].data_ptr(), ldw, N, K, bt.data_ptr(), out.data_ptr(), N)
    torch.cuda.synchronize()
    ctx.synchronize()
    want = oracle_lib.q8_matmul(qx, dx, qw, dw, bias)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))


@pytest.mark.parametrize("N", [130, 8224])
def test_extreme_scales_and_ragged_columns_are_exact(ctx, oracle_lib, cuda, N):
    """Block scales across the fp16 range — subnormal (below 2^-14), tiny normal, large, zero — and a column count that
    leaves a partial 128-column tile: the tensor-core scale products d_x · d_w and the per-block fma stay exact."""
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(N)
    M, K = 257, 320
    qx = rng.integers(-127, 128, (M, K)).astype(np.int8)
    qw = rng.integers(-127, 128, (N, K)).astype(np.int8)
    pick = np.array([3e-8, 5e-6, 6.1e-5, 1e-3, 0.0, 0.5, 40.0], np.float32)
    dx = rng.choice(pick, (M, K // 32)).astype(np.float16).astype(np.float32)
    dw = rng.choice(pick, (N, K // 32)).astype(np.float16).astype(np.float32)
    ldx, ldw = (M + 127) // 128 * 128, (N + 3) // 4 * 4
    dxt = np.zeros((K // 32, ldx), np.float32)
    dxt[:, :M] = dx.T
    dwt = np.zeros((K // 32, ldw), np.float32)
    dwt[:, :N] = dw.T
    dev = [torch.from_numpy(a).cuda() for a in (qx.astype(np.float16), qw.astype(np.float16), dxt, dwt)]
    ldo = ldw + 8
    out = torch.full((M, ldo), float("nan"), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.gemm(ctx, dev[0].data_ptr(), dev[2].data_ptr(), ldx, M, dev[1].data_ptr(), dev[3].data_ptr(), ldw,
                        N, K, None, out.data_ptr(), ldo)
    torch.cuda.synchronize()
    ctx.synchronize()
    want = oracle_lib.q8_matmul(qx, dx, qw, dw)
    got = out.cpu().numpy()
    assert np.array_equal(bits(got[:, :N]), bits(want))
    assert np.all(np.isnan(got[:, (N + 3) // 4 * 4:]))   # stores move whole 16-byte chunks: nothing past them


def test_residual_epilogue_is_exact(ctx, oracle_lib, cuda):
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(21)
    M, N, K = 300, 768, 768
    qx, qw, dx, dw, ldx, ldw, dev = _device_operands(torch, rng, M, N, K)
    h = rng.normal(size=(M, N)).astype(np.float32)
    ht = torch.from_numpy(h).cuda()
    laya_b200.Q8_0.gemm_fused(ctx, laya_b200.Q8_0.RESIDUAL, dev["qx"].data_ptr(), dev["dx"].data_ptr(), ldx, M,
                              dev["qw"].data_ptr(), dev["dw"].data_ptr(), ldw, N, K, None, ht.data_ptr(), N, None,
                              None, 0)
    torch.cuda.synchronize()
    want = h + oracle_lib.q8_matmul(qx, dx, qw, dw)
    assert np.array_equal(bits(ht.cpu().numpy()), bits(want))


def geglu_rows(N):
    I = N // 2
    order = []
    for g in range(N // 64):
        order += list(range(32 * g, 32 * g + 32)) + list(range(I + 32 * g, I + 32 * g + 32))
    return np.array(order)


@pytest.mark.parametrize("M,I", [(300, 1152), (77, 96)])
def test_geglu_epilogue_is_exact(ctx, oracle_lib, cuda, M, I):
    """Wi product → GeGLU (ModernBertEncoder.GeGlu) → the next projection's quantizer, fused: codes and scales equal
    the oracle's separate steps bit for bit."""
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(M + I)
    N, K = 2 * I, 768
    qx, qw, dx, dw, ldx, ldw, dev = _device_operands(torch, rng, M, N, K, scale=0.0002)
    perm = geglu_rows(N)
    dwp = np.zeros((K // 32, ldw), np.float32)
    dwp[:, :N] = dw[perm].T
    qwp = torch.from_numpy(np.ascontiguousarray(qw[perm]).astype(np.float16)).cuda()
    dwpt = torch.from_numpy(dwp).cuda()
    qout = torch.zeros((M, I), dtype=torch.float16, device="cuda")
    qsc = torch.zeros((I // 32, ldx), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.gemm_fused(ctx, laya_b200.Q8_0.GEGLU, dev["qx"].data_ptr(), dev["dx"].data_ptr(), ldx, M,
                              qwp.data_ptr(), dwpt.data_ptr(), ldw, N, K, None, None, 0, qout.data_ptr(),
                              qsc.data_ptr(), ldx)
    torch.cuda.synchronize()
    wide = oracle_lib.q8_matmul(qx, dx, qw, dw)
    act = oracle_lib.geglu(wide)
    wq, wd = oracle_lib.q8_quantize_activations(act)
    assert np.array_equal(codes(qout), wq)
    assert np.array_equal(bits(qsc.cpu().numpy()[:, :M].T), bits(wd))


@pytest.mark.parametrize("M,I", [(300, 9216), (77, 160)])
def test_swiglu_epilogue_is_exact(ctx, oracle_lib, cuda, M, I):
    """The decoder's [gate | up] product → silu(gate) · up (DecoderKernels.SiluMultiply) → the down projection's
    quantizer, fused (weight rows in [32 gate | 32 up] groups): codes and scales equal the oracle's separate steps."""
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(M + I + 1)
    N, K = 2 * I, 256
    qx, qw, dx, dw, ldx, ldw, dev = _device_operands(torch, rng, M, N, K, scale=0.0002)
    perm = geglu_rows(N)            # the same grouping: 32 rows of the first half, then the matching 32 of the second
    dwp = np.zeros((K // 32, ldw), np.float32)
    dwp[:, :N] = dw[perm].T
    qwp = torch.from_numpy(np.ascontiguousarray(qw[perm]).astype(np.float16)).cuda()
    dwpt = torch.from_numpy(dwp).cuda()
    qout = torch.zeros((M, I), dtype=torch.float16, device="cuda")
    qsc = torch.zeros((I // 32, ldx), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.gemm_fused(ctx, laya_b200.Q8_0.SWIGLU, dev["qx"].data_ptr(), dev["dx"].data_ptr(), ldx, M,
                              qwp.data_ptr(), dwpt.data_ptr(), ldw, N, K, None, None, 0, qout.data_ptr(),
                              qsc.data_ptr(), ldx)
    torch.cuda.synchronize()
    wide = oracle_lib.q8_matmul(qx, dx, qw, dw)
    act = np.empty((M, I), np.float32)
    oracle_lib.lib().lo_silu_multiply(np.ascontiguousarray(wide), M, I, act)
    wq, wd = oracle_lib.q8_quantize_activations(act)
    assert np.array_equal(codes(qout), wq)
    assert np.array_equal(bits(qsc.cpu().numpy()[:, :M].T), bits(wd))


def test_relu_epilogue_is_exact(ctx, oracle_lib, cuda):
    torch = cuda
    import laya_b200
    rng = np.random.default_rng(31)
    M, N, K = 200, 3072, 768
    qx, qw, dx, dw, ldx, ldw, dev = _device_operands(torch, rng, M, N, K)
    bias = rng.normal(size=N).astype(np.float32)
    bt = torch.from_numpy(bias).cuda()
    qout = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    qsc = torch.zeros((N // 32, ldx), dtype=torch.float32, device="cuda")
    laya_b200.Q8_0.gemm_fused(ctx, laya_b200.Q8_0.RELU, dev["qx"].data_ptr(), dev["dx"].data_ptr(), ldx, M,
                              dev["qw"].data_ptr(), dev["dw"].data_ptr(), ldw, N, K, bt.data_ptr(), None, 0,
                              qout.data_ptr(), qsc.data_ptr(), ldx)
    torch.cuda.synchronize()
    act = oracle_lib.relu(oracle_lib.q8_matmul(qx, dx, qw, dw, bias))
    wq, wd = oracle_lib.q8_quantize_activations(act)
    assert np.array_equal(codes(qout), wq)
    assert np.array_equal(bits(qsc.cpu().numpy()[:, :M].T), bits(wd))


def test_short_input_is_an_argument_error(ctx):
    """PackedMatrixQ8_0.Multiply throws ArgumentException on a short span (PackedMatrixQ8_0.cs:227-229)."""
    import laya_b200
    m = laya_b200.PackedMatrixQ8_0(ctx, "short", weight=np.ones((64, 64), np.float32))
    with pytest.raises(laya_b200.LayaArgumentError):
        m.multiply(np.ones(64 * 2 - 1, np.float32), 2)
    with pytest.raises(laya_b200.LayaArgumentError):
        laya_b200.PackedMatrixQ8_0(ctx, "bad", weight=np.ones((64, 40), np.float32))
