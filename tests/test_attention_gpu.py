"""Parity of the CUDA windowed attention with the reference semantics."""
import math

import numpy as np
import pytest
import torch

from oracle.attention import local_attention as oracle_attention

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import mergenet_b200  # noqa: F401
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _clean_status():
    """Each case starts with a clear (sticky) attention status word."""
    if torch.cuda.is_available():
        import mergenet_b200
        mergenet_b200.attention.attention_status(torch.device("cuda", 0), reset=True)
    yield


def reference_bhnd(q, k, v, bias, window):
    """The reference test's fp32 restatement (tests/test_biased_local_attention.py:17-29)."""
    q32, k32, v32 = q.float(), k.float(), v.float()
    scores = q32 @ k32.transpose(-1, -2) / math.sqrt(q.shape[-1])
    if bias is not None:
        scores = scores + bias.float()[:, None, None, :]
    if window >= 0:
        tokens = q.shape[-2]
        pos = torch.arange(tokens, device=q.device)
        allowed = (pos[:, None] - pos[None, :]).abs() <= window
        scores = scores.masked_fill(~allowed.view(1, 1, tokens, tokens), float("-inf"))
    return torch.softmax(scores, dim=-1) @ v32


def test_attention_matches_reference_naive(dev, golden_dir):
    """The tensor-core kernel against the reference's own unfold
    implementations (naive_unbiased_local_attention /
    naive_biased_local_attention, run by make_golden.py on the head_dim-64
    case [2, 40, 4, 64], window 16).  Those take a pre-scaled q, so the
    softmax scale is 1 here; the fp32 fixture inputs go in as fp16, as the
    reference casts them for its FlashAttention call (bias_local_attn.py:
    533-537, :357-362), and the bias is rounded to fp16 like its extra
    column."""
    from mergenet_b200.attention import _launch
    g = np.load(golden_dir / "attention.npz")
    i = 1
    assert g[f"q{i}"].shape[-1] == 64
    q, k, v, bias = (torch.from_numpy(g[f"{n}{i}"]).to(dev).half() for n in ("q", "k", "v", "bias"))
    w = int(g[f"window{i}"])
    u = _launch(q, k, v, None, w, False, 1.0, torch.float32)
    b = _launch(q, k, v, bias, w, False, 1.0, torch.float32)
    np.testing.assert_allclose(u.cpu().numpy(), g[f"unbiased{i}"], rtol=5e-3, atol=5e-3)
    np.testing.assert_allclose(b.cpu().numpy(), g[f"biased{i}"], rtol=5e-3, atol=5e-3)
    assert mn_status(dev) == 0


def mn_status(dev):
    import mergenet_b200 as mn
    return mn.attention.attention_status(dev)


def test_fp32_inputs_take_the_reference_fp16_cast(dev):
    """fp32 q/k/v are cast to fp16 before the kernel, as the reference does
    (bias_local_attn.py:533-537); the result equals the oracle on the
    fp16-rounded inputs, and the fp32 output dtype is kept."""
    import mergenet_b200 as mn
    torch.manual_seed(9)
    q = torch.randn(2, 6, 97, 64, device=dev) * 0.4
    k = torch.randn_like(q) * 0.4
    v = torch.randn_like(q)
    out = mn.unbiased_local_attention(q, k, v, 16)
    assert out.dtype == torch.float32
    r = [t.half().float().transpose(1, 2).cpu().numpy() for t in (q, k, v)]
    exp = oracle_attention(*r, 16)
    np.testing.assert_allclose(out.transpose(1, 2).cpu().numpy(), exp, rtol=5e-3, atol=5e-3)
    bias = torch.randn(2, 97, device=dev) * 0.3
    outb = mn.biased_local_attention(q, k, v, bias, 16, input_layout="BHND")
    expb = oracle_attention(*r, 16, bias=bias.half().float().cpu().numpy())
    np.testing.assert_allclose(outb.transpose(1, 2).cpu().numpy(), expb, rtol=5e-3, atol=5e-3)
    assert mn_status(dev) == 0


@pytest.mark.parametrize("layout", ["BHND", "BNHD"])
@pytest.mark.parametrize("tokens,heads,window", [(11, 3, 2), (3, 5, 1), (11, 3, -1)])
def test_biased_parity(dev, layout, tokens, heads, window):
    """tests/test_biased_local_attention.py:32-63 (forward, fp16)."""
    import mergenet_b200 as mn
    torch.manual_seed(20260809)
    batch, dim = 2, 64  # the reference test uses 16; the kernels here take head_dim 64
    q = torch.randn(batch, heads, tokens, dim, device=dev, dtype=torch.float16) * 0.25
    k = torch.randn_like(q) * 0.25
    v = torch.randn_like(q)
    bias = torch.randn(batch, tokens, device=dev, dtype=torch.float16) * 0.25
    if layout == "BHND":
        args = (q, k, v)
    else:
        args = tuple(t.transpose(1, 2).contiguous() for t in (q, k, v))
    out = mn.biased_local_attention(*args, bias, local_window=window, x_dtype=torch.float16, input_layout=layout)
    out_bhnd = out if layout == "BHND" else out.transpose(1, 2)
    expected = reference_bhnd(q, k, v, bias, window)
    # the reference gate allows 1.5e-2; P is rounded to fp16 for P.V as FlashAttention does
    torch.testing.assert_close(out_bhnd.float(), expected, atol=5e-3, rtol=5e-3)


def test_unbiased_parity_layouts(dev):
    import mergenet_b200 as mn
    torch.manual_seed(3)
    q = torch.randn(2, 40, 4, 64, device=dev, dtype=torch.float16) * 0.3
    k = torch.randn_like(q) * 0.3
    v = torch.randn_like(q)
    out = mn.unbiased_local_attention(q, k, v, 16)
    exp = reference_bhnd(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None, 16).transpose(1, 2)
    # head_dim 64 runs on the tensor cores with P rounded to fp16 (as FlashAttention does)
    torch.testing.assert_close(out.float(), exp, atol=5e-3, rtol=5e-3)
    out2 = mn.unbiased_local_attention(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(),
                                       v.transpose(1, 2).contiguous(), 16)
    torch.testing.assert_close(out2.transpose(1, 2).float(), exp, atol=5e-3, rtol=5e-3)
    assert mn.attention.attention_status(dev) == 0


def test_locality(dev):
    """tests/test_biased_local_attention.py:87-113."""
    import mergenet_b200 as mn
    batch, heads, tokens, dim = 1, 3, 11, 64
    window, target = 2, 5
    q = torch.randn(batch, heads, tokens, dim, device=dev, dtype=torch.float16)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    bias = torch.randn(batch, tokens, device=dev, dtype=torch.float16)

    def run(value):
        return mn.biased_local_attention(q, k, value, bias, window, input_layout="BHND")

    base = run(v)
    inside = v.clone()
    inside[:, :, target + 1] += 1
    outside = v.clone()
    outside[:, :, target + window + 2] += 1
    assert (run(inside)[:, :, target] - base[:, :, target]).abs().max().item() > 1e-4
    assert (run(outside)[:, :, target] - base[:, :, target]).abs().max().item() <= 1e-6


def test_ambiguous_layout_rejected(dev):
    import mergenet_b200 as mn
    amb = torch.randn(1, 4, 4, 64, device=dev, dtype=torch.float16)
    with pytest.raises(ValueError):
        mn.biased_local_attention(amb, amb, amb, torch.zeros(1, 4, device=dev, dtype=torch.float16), 1)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_local_block_attention_cls_global(dev, dtype):
    """LocalAttention core at the canonical shape: packed qkv [B, 785, 3*384],
    window 16, CLS row global (bias_local_attn.py:687-721)."""
    import mergenet_b200 as mn
    torch.manual_seed(7)
    b, n, h, d = 4, 785, 6, 64
    qkv = (torch.randn(b, n, 3 * h * d, device=dev) * 0.5).to(dtype)
    out = mn.local_attention_packed(qkv, h, 16, cls_global=True)
    view = qkv.view(b, n, 3, h, d)
    q, k, v = (view[:, :, i].transpose(1, 2) for i in range(3))
    exp = reference_bhnd(q, k, v, None, 16)
    cls = torch.softmax(q[:, :, :1].float() @ k.float().transpose(-1, -2) / 8.0, -1) @ v.float()
    exp[:, :, :1] = cls
    exp = exp.transpose(1, 2).reshape(b, n, h * d)
    tol = 2e-2 if dtype == torch.bfloat16 else 5e-3
    torch.testing.assert_close(out.float(), exp, atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype,biased,cls", [(torch.float16, True, False), (torch.bfloat16, False, True),
                                              (torch.float16, False, True), (torch.float16, True, True)])
def test_window_many_tiles_per_cta(dev, dtype, biased, cls):
    """Window 16 at 785 tokens with more (tile, head, image) work items than
    resident CTAs (12 x 6 x 7 = 504), so each CTA walks several tiles and
    fetches the next one's rows while finishing the current one."""
    import mergenet_b200 as mn
    torch.manual_seed(11 + int(biased) + 2 * int(cls))
    b, n, h, d = 12, 785, 6, 64
    qkv = (torch.randn(b, n, 3 * h * d, device=dev) * 0.5).to(dtype)
    bias = (torch.rand(b, n, device=dev) * 3 + 0.5).log() if biased else None
    out = mn.local_attention_packed(qkv, h, 16, cls_global=cls, bias=bias)
    view = qkv.view(b, n, 3, h, d)
    q, k, v = (view[:, :, i].transpose(1, 2) for i in range(3))
    exp = reference_bhnd(q, k, v, bias.to(dtype) if biased else None, 16)
    if cls:
        logits = q[:, :, :1].float() @ k.float().transpose(-1, -2) / 8.0
        if biased:
            logits = logits + bias.to(dtype).float()[:, None, None, :]
        exp[:, :, :1] = torch.softmax(logits, -1) @ v.float()
    exp = exp.transpose(1, 2).reshape(b, n, h * d)
    tol = 2e-2 if dtype == torch.bfloat16 else 5e-3
    torch.testing.assert_close(out.float(), exp, atol=tol, rtol=tol)
    assert mn.attention.attention_status(dev) == 0


@pytest.mark.parametrize("dtype,biased,out_dtype", [(torch.float16, True, None), (torch.bfloat16, False, None),
                                                    (torch.float16, False, torch.float32)])
def test_full_attention_many_tiles(dev, dtype, biased, out_dtype):
    """Every key of 393, with more (tile, head, image) items than CTAs
    (40 x 6 x 4 = 960): each CTA walks several images and heads, loading the
    next one's K and V while the current one's tiles run."""
    import mergenet_b200 as mn
    torch.manual_seed(5 + int(biased))
    b, n, h, d = 40, 393, 6, 64
    qkv = (torch.randn(b, n, 3 * h * d, device=dev) * 0.5).to(dtype)
    size = torch.rand(b, n, device=dev) * 3 + 0.05
    bias = size.log() if biased else None
    out = mn.local_attention_packed(qkv, h, -1, cls_global=False, bias=bias, out_dtype=out_dtype)
    q, k, v = qkv.view(b, n, 3, h, d).permute(2, 0, 3, 1, 4).unbind(0)
    mask = bias.to(dtype).float()[:, None, None, :] if biased else None
    exp = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=mask)
    tol = 2e-2 if dtype == torch.bfloat16 else 5e-3
    torch.testing.assert_close(out.float(), exp.transpose(1, 2).reshape(b, n, h * d), atol=tol, rtol=tol)
    assert mn.attention.attention_status(dev) == 0


@pytest.mark.parametrize("tokens,window,biased", [(785, 17, False), (785, 40, True), (300, 100, False),
                                                   (131, 70, True)])
def test_wide_window_multi_block(dev, tokens, window, biased):
    """Windows wider than one 160-key block run as several key blocks with an
    online softmax; the last query tile has padding rows whose window starts
    past the current block."""
    import mergenet_b200 as mn
    torch.manual_seed(tokens + window)
    b, h, d = 2, 6, 64
    qkv = (torch.randn(b, tokens, 3 * h * d, device=dev) * 0.5).half()
    bias = (torch.rand(b, tokens, device=dev) * 3 + 0.5).log() if biased else None
    out = mn.local_attention_packed(qkv, h, window, cls_global=False, bias=bias)
    view = qkv.view(b, tokens, 3, h, d)
    q, k, v = (view[:, :, i].transpose(1, 2) for i in range(3))
    exp = reference_bhnd(q, k, v, bias.half() if biased else None, window)
    exp = exp.transpose(1, 2).reshape(b, tokens, h * d)
    torch.testing.assert_close(out.float(), exp, atol=5e-3, rtol=5e-3)
    assert mn.attention.attention_status(dev) == 0


def test_config3_biased_block_against_oracle(dev):
    """Config 3 shape family (785 tokens, 6x64, window 16, per-key bias) at a
    batch the float64 oracle finishes quickly."""
    import mergenet_b200 as mn
    from inputs import attention_inputs
    q, k, v, bias = attention_inputs(0, 2, 785, 6, 64)
    tq, tk, tv, tb = (torch.from_numpy(t).to(dev) for t in (q, k, v, bias))
    out = mn.biased_local_attention(tq, tk, tv, tb, 16, input_layout="BNHD")
    exp = oracle_attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), 16,
                           bias=bias.astype(np.float32))
    err = np.abs(out.float().cpu().numpy() - exp).max() / np.abs(exp).max()
    assert err <= 1e-2


@pytest.mark.parametrize("dtype,out_dtype", [(torch.float16, torch.float32), (torch.bfloat16, torch.bfloat16),
                                             (torch.float16, torch.float16)])
@pytest.mark.parametrize("nq,nk", [(393, 785), (128, 128), (9, 200), (300, 17)])
def test_cross_attention(dev, dtype, out_dtype, nq, nk):
    """Recovery cross-attention core (model.py:173-188): 393 carriers over 785
    tokens, plus ragged query / key counts (partial tiles, one short block)."""
    import mergenet_b200 as mn
    torch.manual_seed(nq * 7 + nk)
    b, h, d = 3, 6, 64
    q = (torch.randn(b, nq, h, d, device=dev) * 0.5).to(dtype)
    k = (torch.randn(b, nk, h, d, device=dev) * 0.5).to(dtype)
    v = torch.randn(b, nk, h, d, device=dev).to(dtype)
    out = mn.cross_attention(q, k, v, out_dtype=out_dtype)
    exp = torch.softmax(q.float().transpose(1, 2) @ k.float().transpose(1, 2).transpose(-1, -2) / 8.0, -1) \
        @ v.float().transpose(1, 2)
    exp = exp.transpose(1, 2)
    tol = 2e-2 if torch.bfloat16 in (dtype, out_dtype) else 5e-3
    torch.testing.assert_close(out.float(), exp, atol=tol, rtol=tol)
    assert mn.attention.attention_status(dev) == 0


def test_cross_attention_strided_projection_views(dev):
    """q/k/v as head views of [B, N, 384] projections, fp32 context out."""
    import mergenet_b200 as mn
    torch.manual_seed(5)
    b = 2
    qp = torch.randn(b, 393, 384, device=dev).half()
    kvp = torch.randn(b, 785, 768, device=dev).half()
    k, v = kvp[..., :384].view(b, 785, 6, 64), kvp[..., 384:].view(b, 785, 6, 64)
    out = mn.cross_attention(qp.view(b, 393, 6, 64), k, v, out_dtype=torch.float32)
    exp = torch.nn.functional.scaled_dot_product_attention(
        qp.view(b, 393, 6, 64).transpose(1, 2).float(), k.transpose(1, 2).float(), v.transpose(1, 2).float())
    torch.testing.assert_close(out, exp.transpose(1, 2), atol=5e-3, rtol=5e-3)


@pytest.mark.parametrize("n", [393, 400, 401, 257, 256, 130, 17, 1])
def test_latent_proportional_attention(dev, n):
    """The latent blocks' ToMe attention (opentome/timm/tome.py:44-58):
    every key, plus log(size) per key, against SDPA with the float mask."""
    import mergenet_b200 as mn
    torch.manual_seed(n)
    b, h, d = 3, 6, 64
    qkv = (torch.randn(b, n, 3 * h * d, device=dev) * 0.5).half()
    size = torch.rand(b, n, device=dev) * 3 + 0.05
    out = mn.local_attention_packed(qkv, h, -1, cls_global=False, bias=size.log())
    q, k, v = qkv.view(b, n, 3, h, d).permute(2, 0, 3, 1, 4).unbind(0)
    exp = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                           attn_mask=size.log().half().float()[:, None, None, :])
    torch.testing.assert_close(out.float(), exp.transpose(1, 2).reshape(b, n, h * d), atol=5e-3, rtol=5e-3)
    assert mn.attention.attention_status(dev) == 0


@pytest.mark.parametrize("rows,y,dtype", [(785 * 3, True, torch.float16), (393 * 2, False, torch.float16),
                                          (7, True, torch.float16), (785 * 2, True, torch.bfloat16)])
def test_add_layernorm(dev, rows, y, dtype):
    from mergenet_b200.model import add_layernorm
    torch.manual_seed(rows)
    x = torch.randn(rows, 384, device=dev) * 3
    yy = torch.randn(rows, 384, device=dev).to(dtype) if y else None
    ln = torch.nn.LayerNorm(384, eps=1e-6).to(dev)
    torch.nn.init.normal_(ln.weight)
    torch.nn.init.normal_(ln.bias)
    s = x + (yy.float() if y else 0)
    xo = torch.empty_like(x)
    _, h, raw = add_layernorm(x, yy, ln, x_out=xo, want_raw=True, dtype=dtype)
    assert torch.equal(xo, s)
    assert torch.equal(raw, s.to(dtype))
    tol = 2e-3 if dtype == torch.float16 else 1.6e-2
    torch.testing.assert_close(h.float(), ln(s).to(dtype).float(), atol=tol, rtol=tol)


@pytest.mark.parametrize("batch,tokens", [(3, 785), (1, 2), (2, 1)])
def test_embed_layernorm(dev, batch, tokens):
    """Position embedding + CLS row into the fp32 stream, fused with norm1:
    the sum is bit-exact with PyTorch's fp32 add, the LayerNorm within fp16
    output rounding."""
    from mergenet_b200.model import embed_layernorm
    torch.manual_seed(tokens)
    emb = (torch.randn(batch, tokens - 1, 384, device=dev) * 2).half()
    pos = torch.randn(tokens, 384, device=dev) * 0.02
    cls = torch.randn(384, device=dev) * 1e-3
    ln = torch.nn.LayerNorm(384, eps=1e-6).to(dev)
    torch.nn.init.normal_(ln.weight)
    torch.nn.init.normal_(ln.bias)
    want = torch.cat([cls.expand(batch, 1, -1), emb.float()], 1) + pos
    x, h = embed_layernorm(emb, pos, cls, ln)
    assert torch.equal(x, want)
    torch.testing.assert_close(h.float(), ln(want).half().float(), atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("b,c,hw,p", [(3, 3, 224, 8), (2, 3, 32, 8), (1, 2, 48, 16)])
def test_patch_unfold_exact(dev, b, c, hw, p):
    """The patch unfold equals PyTorch's permuted fp16 copy bit for bit."""
    from mergenet_b200 import _lib as L
    g = torch.Generator(device=dev).manual_seed(hw + p)
    img = torch.randn(b, c, hw, hw, device=dev, generator=g)
    gh = hw // p
    out = torch.empty(b, gh, gh, c, p, p, device=dev, dtype=torch.float16)
    L.check(L.lib().mn_patch_unfold(b, c, hw, hw, p, L.ptr(img), L.ptr(out), L.stream_of(img)), "unfold")
    want = img.view(b, c, gh, p, gh, p).permute(0, 2, 4, 1, 3, 5).half()
    assert torch.equal(out, want)


def test_window_attention_matches_flash_attention(dev):
    """The reference's windowed attention IS FlashAttention-2's
    flash_attn_func(window_size=(w, w)) (bias_local_attn.py:560-567); the
    flash_attn library is installed, so compare with it directly on the
    canonical shape (785 tokens, 6 heads of 64, window 16), q/k/v read from
    the packed projection."""
    fa = pytest.importorskip("flash_attn")
    import mergenet_b200 as mn
    torch.manual_seed(21)
    b, n, h, d = 4, 785, 6, 64
    qkv = (torch.randn(b, n, 3 * h * d, device=dev) * 0.5).half()
    view = qkv.view(b, n, 3, h, d)
    want = fa.flash_attn_func(view[:, :, 0], view[:, :, 1], view[:, :, 2], window_size=(16, 16))
    got = mn.local_attention_packed(qkv, h, 16, cls_global=False).view(b, n, h, d)
    torch.testing.assert_close(got.float(), want.float(), atol=5e-3, rtol=5e-3)


def test_bounded_wait_gives_up_and_the_context_survives(dev):
    """A tensor-core wait that nothing completes ends after its limit with
    MN_STATUS_TC_TIMEOUT in the status word (mn_tc_wait_selftest: TMEM
    allocated and freed as in the kernels), and the next attention call on
    the same context runs clean and correct."""
    import time
    from mergenet_b200 import _lib as L
    import mergenet_b200 as mn
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.perf_counter()
    L.check(L.lib().mn_tc_wait_selftest(L.ptr(status), 20.0, L.stream_of(status)), "mn_tc_wait_selftest")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) & L.MN_STATUS_TC_TIMEOUT
    assert elapsed < 5.0
    torch.manual_seed(2)
    qkv = (torch.randn(2, 785, 1152, device=dev) * 0.5).half()
    out = mn.local_attention_packed(qkv, 6, 16, cls_global=True)
    view = qkv.view(2, 785, 3, 6, 64)
    q, k, v = (view[:, :, i].transpose(1, 2) for i in range(3))
    exp = reference_bhnd(q, k, v, None, 16)
    exp[:, :, :1] = torch.softmax(q[:, :, :1].float() @ k.float().transpose(-1, -2) / 8.0, -1) @ v.float()
    torch.testing.assert_close(out.float(), exp.transpose(1, 2).reshape(2, 785, 384), atol=5e-3, rtol=5e-3)
    assert mn.attention.attention_status(dev) == 0


@pytest.mark.parametrize("b,nq,nk,h,dtype,biased", [
    (48, 393, 393, 6, torch.float16, True),    # latent shape, several tiles per query stream
    (48, 393, 393, 6, torch.bfloat16, True),
    (48, 393, 785, 6, torch.float16, False),   # cross shape, several tiles per query stream
    (1, 1000, 2000, 2, torch.bfloat16, False),
    (300, 9, 64, 1, torch.float16, False),     # one key block, many tiny items
])
def test_warp_specialised_many_items(dev, b, nq, nk, h, dtype, biased):
    """The warp-specialised kernel (latent and cross) when each of its query
    streams walks many (tile, head, image) items: Q stages and the K/V / S
    rings wrap many times.  Checked against an fp32 restatement, and run
    twice to check the result is bit-for-bit repeatable."""
    import mergenet_b200 as mn
    g = torch.Generator(device="cpu").manual_seed(b * 1000 + nq + nk)
    q = (torch.randn(b, nq, h, 64, generator=g) * 0.5).to(dev, dtype)
    k = (torch.randn(b, nk, h, 64, generator=g) * 0.5).to(dev, dtype)
    v = torch.randn(b, nk, h, 64, generator=g).to(dev, dtype)
    # the bias as fp32, or in the operand dtype (the kernel reads either)
    bias = (torch.rand(b, nk, generator=g) * 3 + 0.05).log().to(dev, torch.float32 if b == 48 and
                                                                  dtype == torch.float16 else dtype) \
        if biased else None
    if biased:
        qkv = torch.stack([q, k, v], dim=2).reshape(b, nq, 3 * h * 64)
        run = lambda: mn.local_attention_packed(qkv, h, -1, cls_global=False, bias=bias).view(b, nq, h, 64)
    else:
        run = lambda: mn.cross_attention(q, k, v)
    out1, out2 = run(), run()
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), k.float()) / 8.0
    if biased:
        s = s + bias.to(dtype).float()[:, None, None, :]
    exp = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), v.float())
    tol = 2e-2 if dtype == torch.bfloat16 else 5e-3
    torch.testing.assert_close(out1.float(), exp, atol=tol, rtol=tol)
    assert torch.equal(out1, out2)
    assert mn.attention.attention_status(dev) == 0


def test_empty_batch_attention(dev):
    """Zero images: every attention entry point returns an empty result and
    launches nothing (the reference returns empty tensors for an empty batch)."""
    import mergenet_b200 as mn
    qkv = torch.zeros(0, 785, 1152, device=dev, dtype=torch.float16)
    assert mn.local_attention_packed(qkv, 6, 16, cls_global=True).shape == (0, 785, 384)
    assert mn.local_attention_packed(qkv[:, :393], 6, -1, cls_global=False,
                                     bias=torch.zeros(0, 393, device=dev)).shape == (0, 393, 384)
    q = torch.zeros(0, 393, 6, 64, device=dev, dtype=torch.float16)
    kv = torch.zeros(0, 785, 6, 64, device=dev, dtype=torch.float16)
    assert mn.cross_attention(q, kv, kv).shape == (0, 393, 6, 64)
    assert mn.attention.attention_status(dev) == 0


@pytest.mark.parametrize("rows,y,dtype", [(393 * 3, True, torch.float16), (393 * 2, True, torch.bfloat16),
                                          (5, False, torch.float16)])
def test_add_layernorm_f32(dev, rows, y, dtype):
    """The latent encoder's final norm: LayerNorm(x + y) in fp32 (autocast runs
    layer_norm in fp32, model.py:1195-1198), fused with the residual add."""
    from mergenet_b200.model import add_layernorm_f32
    torch.manual_seed(rows)
    x = torch.randn(rows, 384, device=dev) * 3
    yy = torch.randn(rows, 384, device=dev).to(dtype) if y else None
    ln = torch.nn.LayerNorm(384, eps=1e-6).to(dev)
    torch.nn.init.normal_(ln.weight)
    torch.nn.init.normal_(ln.bias)
    out = add_layernorm_f32(x, yy, ln)
    exp = torch.nn.functional.layer_norm(x + (yy.float() if y else 0), (384,), ln.weight, ln.bias, ln.eps)
    assert out.dtype == torch.float32
    torch.testing.assert_close(out, exp, atol=2e-5, rtol=2e-5)
