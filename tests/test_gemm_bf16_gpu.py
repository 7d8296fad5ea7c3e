"""The bf16 tensor-core product of the training step against torch (fp32 products of the same bf16 values).

The three layouts the training step uses: y = x·Wᵀ (both K-major), dx = dy·W (W read N-contiguous),
dW += dyᵀ·x (both read with the output index contiguous); epilogues bf16, fp32 and fp32 accumulate, with bias.
"""
import numpy as np
import pytest

from conftest import max_rel

pytestmark = pytest.mark.gpu

# CTA-pair tilings: (1000, 2304) every tile split along N (36 tiles, 74 pairs); (4096, 1152) a narrow last column and
# a split last round; (20480, 768) three full rounds and a split fourth; (2304, 1152, 4096) a narrow last column with
# the K split of accumulating outputs; (72, 96) and (136, 200) the one-CTA kernels and a single pair tile.
SHAPES = [(1000, 2304, 768), (304, 768, 1152), (72, 96, 128), (136, 200, 72), (4096, 1152, 768), (20480, 768, 256),
          (2304, 1152, 4096)]
LAYOUTS = [(0, 0), (0, 1), (1, 1)]


@pytest.fixture(scope="module")
def ctx(cuda):
    import laya_b200
    c = laya_b200.Context(laya_b200.base_desc(max_tokens=256, max_items=4, max_markers=16))
    c.set_stream(cuda.cuda.current_stream().cuda_stream)
    yield c
    c.close()


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", LAYOUTS)
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_product_matches_torch(ctx, cuda, M, N, K, a_mn, b_mn, epi):
    torch = cuda
    import laya_b200
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K + 13 * a_mn + 5 * b_mn + epi)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g)
    As = A.t().contiguous() if a_mn else A
    Bs = B.t().contiguous() if b_mn else B
    lda = M if a_mn else K
    ldb = N if b_mn else K
    want = A.float() @ B.float().t() + bias
    if epi == 0:
        out = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    else:
        out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
        if epi == 2:
            base = torch.randn(M, N, device="cuda", generator=g)
            out.copy_(base)
            want = want + base
    laya_b200.api.check(laya_b200.lib().laya_gemm_bf16_device(
        ctx.handle, M, N, K, As.data_ptr(), lda, a_mn, Bs.data_ptr(), ldb, b_mn, bias.data_ptr(), epi, out.data_ptr(), N))
    torch.cuda.synchronize()
    ctx.synchronize()
    err = max_rel(out.float().cpu().numpy(), want.cpu().numpy())
    assert err < (8e-3 if epi == 0 else 2e-5), f"max rel {err:.2e}"


@pytest.mark.parametrize("M,N,K", [(1000, 2304, 768), (136, 200, 72), (304, 96, 1152)])
@pytest.mark.parametrize("a_mn,b_mn", LAYOUTS)
def test_split_product_is_fp32_accurate(ctx, cuda, M, N, K, a_mn, b_mn):
    """hi·hi + lo·hi + hi·lo of bf16 parts reproduces the fp32 product (float64 reference) to ~2^-16 relative, far
    inside bf16's 2^-8: the accurate forward of the fine-tuning step."""
    torch = cuda
    import laya_b200
    g = torch.Generator(device="cuda").manual_seed(M + N + K + a_mn)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(N, K, device="cuda", generator=g)
    bias = torch.randn(N, device="cuda", generator=g)
    want = (A.double() @ B.double().t() + bias.double()).cpu().numpy()
    parts = []
    for X, mn in ((A, a_mn), (B, b_mn)):
        hi = X.to(torch.bfloat16)
        lo = (X - hi.float()).to(torch.bfloat16)
        parts += [(hi.t().contiguous(), lo.t().contiguous()) if mn else (hi, lo)]
    (Ah, Al), (Bh, Bl) = parts
    out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    laya_b200.api.check(laya_b200.lib().laya_gemm_bf16_split_device(
        ctx.handle, M, N, K, Ah.data_ptr(), Al.data_ptr(), M if a_mn else K, a_mn, Bh.data_ptr(), Bl.data_ptr(),
        N if b_mn else K, b_mn, bias.data_ptr(), 1, out.data_ptr(), N))
    torch.cuda.synchronize()
    ctx.synchronize()
    err = max_rel(out.cpu().numpy(), want)
    plain = max_rel((A.to(torch.bfloat16).float() @ B.to(torch.bfloat16).float().t() + bias).cpu().numpy(), want)
    assert err < 1e-4 and err < plain / 50, f"split {err:.2e} vs plain bf16 {plain:.2e}"
