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


@pytest.mark.parametrize("m,n", [(393 * 3, 384), (785 * 2 + 5, 768), (17, 128)])
def test_split_precision_linear_is_fp32_accurate(dev, m, n):
    """The cross-attention's fp32 Linear layers on the split-precision
    tcgen05 GEMM.  Against a float64 product its largest error is within
    3.5x that of PyTorch's IEEE fp32 GEMM (no TF32) on the same operands
    (measured 1.2-2.5x: the operand halves are exact to 2^-22, and the tensor
    cores' fp32 accumulation is not round-to-nearest) -- about 1e-6 of the
    largest output, against about 1e-3 for TF32.  Its fp16-output form is
    within one fp16 ulp of the exact product's rounding, and equal to it for
    almost every output."""
    from mergenet_b200.linear import SplitWeight, layernorm_split, linear_f32_split
    torch.manual_seed(m + n)
    k = 384
    x = torch.randn(m, k, device=dev) * 3 + 0.5
    ln = torch.nn.LayerNorm(k).to(dev)
    torch.nn.init.normal_(ln.weight, 1.0, 0.1)
    torch.nn.init.normal_(ln.bias, 0.0, 0.05)
    lin = torch.nn.Linear(k, n).to(dev)
    hi, lo = layernorm_split(x, ln)
    y = ln(x).detach()
    torch.testing.assert_close((hi.double() + lo.double()) / 256.0, y.double(), rtol=1e-6, atol=1e-7)
    w = SplitWeight(lin.weight, lin.bias)
    got = linear_f32_split(hi, lo, w)
    want = (y.double() @ lin.weight.double().t() + lin.bias.double())
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        fp32 = torch.nn.functional.linear(y, lin.weight, lin.bias).double()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    scale = want.abs().max()
    err_split = ((got.double() - want).abs().max() / scale).item()
    err_fp32 = ((fp32 - want).abs().max() / scale).item()
    assert err_split <= 3.5 * err_fp32 + 1e-7, (err_split, err_fp32)
    half = linear_f32_split(hi, lo, w, out_dtype=torch.float16)
    assert half.dtype == torch.float16
    # against the exact product: half an fp16 ulp of rounding plus the GEMM's
    # own error bound; and equal to the fp16 rounding of the exact product for
    # at least 99% of the outputs (an error of 1e-6 of the largest output
    # decides the rounding of some outputs near zero)
    exact16 = want.float().half()
    mag = want.abs().clamp_min(2.0 ** -14)
    half_ulp = torch.exp2(torch.floor(torch.log2(mag)) - 11)
    bound = half_ulp + (3.5 * err_fp32 + 1e-7) * scale
    assert bool(((half.double() - want).abs() <= bound * 1.0001).all())
    assert (half == exact16).float().mean().item() >= 0.99
    # an fp16-exact A (the attention context) needs no lo plane
    a16 = (torch.randn(m, k, device=dev) * 0.5).half()
    got16 = linear_f32_split(a16, None, w, a_scale=1.0)
    want16 = a16.double() @ lin.weight.double().t() + lin.bias.double()
    assert ((got16.double() - want16).abs().max() / want16.abs().max()).item() <= 2e-6
    from mergenet_b200.linear import gemm_status
    assert gemm_status(dev) == 0


def test_model_cross_attention_ieee_option_agrees(dev):
    """cross_precision="ieee" runs the cross-attention projections as IEEE
    fp32 cuBLAS GEMMs; the default split-precision path agrees with it on
    the recovery output to 1e-3 of the largest value, inside the 2e-3
    feature tolerance (q/k/v are rounded to fp16 for the attention, as in
    the reference, so a 1e-6 difference can move an element by an fp16 ulp)."""
    from mergenet_b200.model import MergeNetSmall
    torch.manual_seed(4)
    m = MergeNetSmall(img_size=32, patch_size=8, num_classes=10, metric_dim=16, local_depth=2, latent_depth=2,
                      local_window=2).init_weights(0)
    torch.nn.init.normal_(m.encode_cross_attention.out_proj.weight, 0, 0.05)
    m = m.to(dev).eval()
    topk_x = torch.randn(3, 393, 384, device=dev)
    x_embed = torch.randn(3, 785, 384, device=dev)
    split = m._cross(topk_x, x_embed)
    m.cross_precision = "ieee"
    ieee = m._cross(topk_x, x_embed)
    assert ((split - ieee).abs().max() / ieee.abs().max()).item() <= 1e-3
