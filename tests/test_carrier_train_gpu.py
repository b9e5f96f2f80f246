"""The carrier block's soft-top-k training terms (model.py:1163-1206) on the
GPU against plain PyTorch restatements of the reference's tensor ops:
the straight-through carrier weights (model.py:1176-1179) and the soft-top-k
auxiliary representation (model.py:1196-1198), forward and backward, and the
gradient they send through ThreTopK to the DTEM masses."""
import numpy as np
import pytest
import torch

from oracle import routing as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import mergenet_b200  # noqa: F401
    return torch.device("cuda", 0)


def ref_aux(x_patches, soft_sel):
    """model.py:1196-1198 as the reference writes it."""
    w = soft_sel / soft_sel.sum(dim=1, keepdim=True).clamp(min=1e-6)
    return (x_patches * w.unsqueeze(-1)).sum(dim=1)


def ref_ste(topk_x_trace, soft_sel, idx):
    """model.py:1176-1179 as the reference writes it."""
    w = torch.gather(soft_sel, 1, idx)
    return topk_x_trace * (1.0 + (w - w.detach())).unsqueeze(-1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_soft_topk_aux_forward_and_backward(dev, dtype):
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(7)
    b, t, c = 3, 785, 384
    x_local = torch.randn(b, t, c, generator=gen).to(dtype)
    sel = torch.rand(b, t - 1, generator=gen)
    sel[2] = 0.0  # an all-zero row: the clamp of the row sum takes over
    g = torch.randn(b, c, generator=gen)
    xd = x_local.to(dev).requires_grad_(True)
    sd = sel.to(dev).requires_grad_(True)
    aux = mn.soft_topk_aux_repr(xd[:, 1:], sd)  # a strided view, as the model passes it
    xr = x_local.double().requires_grad_(True)
    sr = sel.double().requires_grad_(True)
    want = ref_aux(xr[:, 1:], sr)
    np.testing.assert_allclose(aux.detach().cpu().numpy(), want.detach().numpy(), rtol=1e-5, atol=1e-6)
    aux.backward(g.to(dev))
    want.backward(g.double())
    tol = 1e-5 if dtype == torch.float32 else 2e-3
    np.testing.assert_allclose(xd.grad.float().cpu().numpy(), xr.grad.numpy(), rtol=tol, atol=tol * 1e-2)
    gs, want_s = sd.grad.cpu().numpy(), sr.grad.numpy()
    for r in range(b):  # per image: the zero row's gradient is ~1e6 times the others'
        assert np.abs(gs[r] - want_s[r]).max() <= 1e-4 * np.abs(want_s[r]).max(), r
    assert not xd.grad[:, 0].any()  # the CLS row takes no part


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_carrier_ste_forward_and_backward(dev, dtype):
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(8)
    b, n, k, c = 4, 784, 392, 384
    topk = torch.randn(b, k, c, generator=gen).to(dtype)
    sel = torch.rand(b, n, generator=gen)
    idx = torch.stack([torch.randperm(n, generator=gen)[:k] for _ in range(b)])
    g = torch.randn(b, k, c, generator=gen).to(dtype)
    td = topk.to(dev).requires_grad_(True)
    sd = sel.to(dev).requires_grad_(True)
    out = mn.carrier_ste(td, sd, idx.to(dev))
    assert torch.equal(out.detach(), td.detach())  # the forward value is the features themselves
    out.backward(g.to(dev))
    assert torch.equal(td.grad, g.to(dev))
    tr = topk.double().requires_grad_(True)
    sr = sel.double().requires_grad_(True)
    ref_ste(tr, sr, idx).backward(g.double())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    np.testing.assert_allclose(sd.grad.cpu().numpy(), sr.grad.numpy(), rtol=tol, atol=tol)
    # patches that carry nothing get no gradient
    carried = torch.zeros(b, n, dtype=torch.bool)
    carried.scatter_(1, idx, True)
    assert not sd.grad.cpu()[~carried].any()


def test_soft_topk_terms_through_thre_topk(dev):
    """model.py:1163-1206 in training: soft_sel = ThreTopK(masses, k, 30);
    the STE on the carriers and the aux representation both feed the loss.
    The masses' gradient equals the oracle's ThreTopK gradient applied to
    the soft weights' total gradient (from a float64 restatement)."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(9)
    b, n, k, c = 4, 784, 392, 64
    strength = (torch.rand(b, n, generator=gen) * 3 + 0.2)
    x_local = torch.randn(b, n + 1, c, generator=gen)
    g_trace = torch.randn(b, k, c, generator=gen)
    g_aux = torch.randn(b, c, generator=gen)
    st = strength.to(dev).requires_grad_(True)
    xd = x_local.to(dev)
    soft = mn.ThreTopK(st, k, temperature=30.0)
    idx = torch.topk(strength, k, dim=1, largest=True, sorted=False).indices
    topk_x = torch.gather(x_local[:, 1:], 1, idx.unsqueeze(-1).expand(-1, -1, c))
    trace = mn.carrier_ste(topk_x.to(dev), soft, idx.to(dev))
    aux = mn.soft_topk_aux_repr(xd[:, 1:], soft)
    ((trace * g_trace.to(dev)).sum() + (aux * g_aux.to(dev)).sum()).backward()
    # float64 restatement with soft_sel as the leaf, then ThreTopK's gradient
    sr = torch.from_numpy(O.thre_topk(strength.numpy(), k, 30.0)).double().requires_grad_(True)
    ((ref_ste(topk_x.double(), sr, idx) * g_trace.double()).sum() +
     (ref_aux(x_local[:, 1:].double(), sr) * g_aux.double()).sum()).backward()
    want = O.thre_topk_backward(strength.numpy(), k, sr.grad.numpy(), 30.0)
    got = st.grad.cpu().numpy()
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
