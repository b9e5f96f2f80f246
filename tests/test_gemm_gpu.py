"""The tcgen05 GEMM (mn_gemm_f16) against PyTorch's fp16 linear layers."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _clean_status():
    if torch.cuda.is_available():
        from mergenet_b200.linear import gemm_status
        gemm_status(torch.device("cuda", 0), reset=True)
    yield


@pytest.mark.parametrize("m,n,k", [(785 * 3, 1536, 384), (393 * 2, 384, 1536), (785 * 2, 1152, 384),
                                   (127, 128, 64), (1, 256, 128), (4099, 384, 384)])
@pytest.mark.parametrize("gelu", [False, True])
def test_linear_f16_matches_torch(dev, m, n, k, gelu):
    """fp32 accumulation in a different order than cuBLAS: compare within
    fp16 output rounding plus accumulation noise."""
    from mergenet_b200.linear import gemm_status, linear_f16
    g = torch.Generator(device=dev).manual_seed(m + n + k)
    x = torch.randn(m, k, device=dev, generator=g).half()
    w = (torch.randn(n, k, device=dev, generator=g) * k ** -0.5).half()
    b = (torch.randn(n, device=dev, generator=g) * 0.1).half()
    y = linear_f16(x, w, b, gelu=gelu)
    ref = F.linear(x.float(), w.float(), b.float()).half()
    if gelu:
        ref = F.gelu(ref.float()).half()
    torch.cuda.synchronize()
    assert gemm_status(dev) == 0
    torch.testing.assert_close(y.float(), ref.float(), atol=4e-3, rtol=4e-3)


def test_linear_f16_strided_rows_and_no_bias(dev):
    from mergenet_b200.linear import linear_f16
    g = torch.Generator(device=dev).manual_seed(3)
    big = torch.randn(300, 3 * 384, device=dev, generator=g).half()
    x = big[:, 384:768]  # row stride 1152
    w = (torch.randn(384, 384, device=dev, generator=g) * 0.05).half()
    y = linear_f16(x, w, None)
    ref = F.linear(x.float(), w.float()).half()
    torch.testing.assert_close(y.float(), ref.float(), atol=4e-3, rtol=4e-3)


def test_linear_f16_rejects_unsupported(dev):
    from mergenet_b200.linear import linear_f16
    x = torch.randn(8, 100, device=dev).half()
    w = torch.randn(128, 100, device=dev).half()
    with pytest.raises(ValueError):
        linear_f16(x, w)  # K not a multiple of 64


def test_gelu_epilogue_accuracy(dev):
    """GELU of exactly representable fp16 inputs (identity weights) against
    the exact erf form in float64: within half an fp16 ulp of the result plus
    the polynomial's bound 2.3e-5 |x|."""
    import math
    from mergenet_b200.linear import linear_f16
    xs = torch.linspace(-8, 8, 64 * 257, device=dev).half().view(-1, 64)
    w = torch.zeros(128, 64, device=dev, dtype=torch.float16)
    w[:64] = torch.eye(64, device=dev, dtype=torch.float16)
    y = linear_f16(xs, w, None, gelu=True)[:, :64].double().cpu()
    x64 = xs.double().cpu()
    exact = 0.5 * x64 * (1 + torch.erf(x64 / math.sqrt(2)))
    ulp = torch.where(exact.abs() < 6.1e-5, torch.full_like(exact, 5.96e-8),
                      2.0 ** (torch.floor(torch.log2(exact.abs().clamp_min(6.1e-5))) - 10))
    bound = 0.5 * ulp + 2.3e-5 * x64.abs() + 1e-7
    assert bool(((y - exact).abs() <= bound).all()), float(((y - exact).abs() - bound).max())
