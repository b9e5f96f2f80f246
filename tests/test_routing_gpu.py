"""Parity of the CUDA routing path with the reference (fixtures) and the oracle."""
import numpy as np
import pytest
import torch

from conftest import carrier_mismatches, rel_err
from inputs import canonical_r_list, routing_inputs
from oracle import routing as O

pytestmark = pytest.mark.gpu

ROUTE_CASES = ["route_g3x6", "route_g4x4", "route_c1", "route_g48", "route_c2_b128"]


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import mergenet_b200  # noqa: F401  (loads the library; raises if it is missing)
    return torch.device("cuda", 0)


def _case_inputs(g, x_dtype=np.float32, metric_dtype=np.float16):
    grid = tuple(int(v) for v in g["grid"])
    r_list = [int(v) for v in g["r_list"]]
    x, metrics = routing_inputs(int(g["seed"]), int(g["batch"]), grid, int(g["channels"]), int(g["metric_dim"]),
                                layers=len(r_list), metric_dtype=metric_dtype)
    return grid, float(g["radius"]), r_list, x.astype(x_dtype), metrics


def _report_mismatch(got, want, center, margin):
    return [(b, kind, float(margin[b])) for b, kind in carrier_mismatches(got, want, center)]


@pytest.mark.parametrize("name", ROUTE_CASES)
def test_fused_route_matches_reference(dev, golden_dir, name):
    import mergenet_b200 as mn
    g = np.load(golden_dir / f"{name}.npz")
    grid, radius, r_list, x, metrics = _case_inputs(g)
    plan = mn.RoutePlan(grid, radius, r_list, device=dev)
    res = plan(torch.from_numpy(x).to(dev), torch.from_numpy(metrics).to(dev))
    torch.cuda.synchronize()
    assert int(res.status.item()) == 0
    idx = res.topk_idx.cpu().numpy()
    mism = _report_mismatch(idx, g["topk_idx"], g["center"], g["margin"])
    assert not mism, f"carrier mismatch (image, kind, reference rank-k margin): {mism}"
    np.testing.assert_allclose(res.size.cpu().numpy(), g["size"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(res.center.cpu().numpy(), g["center"], rtol=0, atol=2e-3)
    np.testing.assert_allclose(res.topk_size.cpu().numpy(), g["topk_size"], rtol=3e-5, atol=3e-5)
    if "topk_x" in g:
        assert rel_err(res.topk_x.cpu().numpy(), g["topk_x"]) <= 2e-3


@pytest.mark.parametrize("grid,radius,metric_dim", [((4, 5), 2.0, 16), ((6, 7), 3.0, 48), ((5, 6), 3.0, 40)])
def test_fused_route_other_shapes(dev, grid, radius, metric_dim):
    """Shapes off the canonical path, against the oracle: odd grid widths
    (the table-driven transport), an even width whose receiver columns do not
    pair up (the stencil's column pairs with a missing partner), receiver
    in-degree above the unrolled 12 (6x7 at radius 3), and metric widths the
    one-thread-per-donor scorer does not take (16, 48, 40)."""
    import mergenet_b200 as mn
    r_list = canonical_r_list(grid)
    x, metrics = routing_inputs(5, 3, grid, 40, metric_dim)
    ref = O.route_and_gather(x, metrics, r_list, O.Geometry(grid, radius))
    plan = mn.RoutePlan(grid, radius, r_list, device=dev)
    res = plan(torch.from_numpy(x).to(dev), torch.from_numpy(metrics).to(dev))
    mism = carrier_mismatches(res.topk_idx.cpu().numpy(), ref["topk_idx"], ref["center"])
    assert not mism, mism
    np.testing.assert_allclose(res.size.cpu().numpy(), ref["size"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(res.center.cpu().numpy(), ref["center"], rtol=0, atol=2e-3)
    assert rel_err(res.topk_x.cpu().numpy(), ref["topk_x"]) <= 2e-3


def test_fused_route_fp16_tokens(dev, golden_dir):
    """Config-2 storage mode: fp16 tokens in, fp16 carriers out, fp32 math."""
    import mergenet_b200 as mn
    g = np.load(golden_dir / "route_c1.npz")
    grid, radius, r_list, x, metrics = _case_inputs(g)
    x16 = x.astype(np.float16)
    plan = mn.RoutePlan(grid, radius, r_list, device=dev)
    res = plan(torch.from_numpy(x16).to(dev), torch.from_numpy(metrics).to(dev))
    assert not carrier_mismatches(res.topk_idx.cpu().numpy(), g["topk_idx"], g["center"])
    ref = O.route_and_gather(x16.astype(np.float32), metrics, r_list, O.Geometry(grid, radius))
    assert res.topk_x.dtype == torch.float16
    assert rel_err(res.topk_x.float().cpu().numpy(), ref["topk_x"]) <= 1e-2


def test_fused_route_bf16_grid48(dev):
    """Config-5 style: 48x48 grid, bf16 tokens and metrics."""
    import mergenet_b200 as mn
    grid = (48, 48)
    r_list = canonical_r_list(grid)
    x, metrics = routing_inputs(11, 2, grid, 24, 64, layers=6, metric_dtype=np.float32)
    m_bf = torch.from_numpy(metrics).bfloat16()
    x_bf = torch.from_numpy(x).bfloat16()
    plan = mn.RoutePlan(grid, 3.0, r_list, device=dev)
    res = plan(x_bf.to(dev), m_bf.to(dev))
    ref = O.route_and_gather(x_bf.float().numpy(), m_bf.float().numpy(), r_list, O.Geometry(grid, 3.0))
    mism = _report_mismatch(res.topk_idx.cpu().numpy(), ref["topk_idx"], ref["center"],
                            O.carrier_margin(ref["size"], plan.k))
    assert not mism, mism
    assert rel_err(res.topk_x.float().cpu().numpy(), ref["topk_x"]) <= 1e-2


def test_fused_route_is_deterministic(dev, golden_dir):
    import mergenet_b200 as mn
    g = np.load(golden_dir / "route_c1.npz")
    grid, radius, r_list, x, metrics = _case_inputs(g)
    plan = mn.RoutePlan(grid, radius, r_list, device=dev)
    xt, mt = torch.from_numpy(x).to(dev), torch.from_numpy(metrics).to(dev)
    a, b = plan(xt, mt), plan(xt, mt)
    assert torch.equal(a.topk_x, b.topk_x) and torch.equal(a.size, b.size) and torch.equal(a.topk_idx, b.topk_idx)


def test_fused_route_full_batch_properties(dev):
    """Canonical B=256 shard: size-independent invariants (mass conservation,
    carrier set = exact top-k, order by centre, CLS row untouched)."""
    import mergenet_b200 as mn
    grid = (28, 28)
    x, metrics = routing_inputs(3, 256, grid, 384, 64)
    plan = mn.RoutePlan(grid, 3.0, canonical_r_list(grid), device=dev)
    xt, mt = torch.from_numpy(x).to(dev), torch.from_numpy(metrics).to(dev)
    res = plan(xt, mt)
    size = res.size.double()
    # soft merge conserves mass: every layer moves exactly what donors lose
    torch.testing.assert_close(size[:, 1:].sum(1), torch.full_like(size[:, 0], 784.0), rtol=1e-5, atol=1e-3)
    srt = torch.sort(res.size[:, 1:], dim=1, descending=True).values
    kth = srt[:, plan.k - 1:plan.k]
    sel = torch.gather(res.size[:, 1:], 1, res.topk_idx)
    assert bool((sel >= kth).all())
    cen = torch.gather(res.center[:, 1:], 1, res.topk_idx)
    assert bool((cen[:, 1:] >= cen[:, :-1]).all())
    assert torch.equal(res.topk_x[:, 0], xt[:, 0])
    # the whole shard against the oracle: exact carrier sets, order up to
    # float32-tied centres, features within 2e-3
    ref = O.route_and_gather(x, metrics, canonical_r_list(grid), O.Geometry(grid, 3.0))
    mism = _report_mismatch(res.topk_idx.cpu().numpy(), ref["topk_idx"], ref["center"],
                            O.carrier_margin(ref["size"], plan.k))
    assert not mism, mism
    np.testing.assert_allclose(res.size.cpu().numpy(), ref["size"], rtol=3e-5, atol=3e-5)
    same = (res.topk_idx.cpu().numpy() == ref["topk_idx"]).all(1)
    assert rel_err(res.topk_x.cpu().numpy()[same], ref["topk_x"][same]) <= 2e-3


def test_route_budget_fails_closed(dev):
    import mergenet_b200 as mn
    with pytest.raises(RuntimeError):
        mn.RoutePlan((1, 4), 0.5, [1], device=dev)


# ------------------------------------------------------------------ drop-ins
def test_sparse_spatial_score_matches_reference(dev, golden_dir):
    import mergenet_b200 as mn
    g = np.load(golden_dir / "select_g3x5.npz")
    nbr, val = mn.build_patch_spatial_neighbors((3, 5), 2, device=dev)
    a = torch.from_numpy(g["a"]).to(dev)
    b = torch.from_numpy(g["b"]).to(dev)
    ai = torch.from_numpy(g["a_idx"]).to(dev) - 1
    bi = torch.from_numpy(g["b_idx"]).to(dev) - 1
    s, ri, rv = mn.sparse_spatial_score(a, b, nbr, val, ai, bi)
    np.testing.assert_allclose(s.cpu().numpy(), g["scores"], rtol=0, atol=2e-5)
    np.testing.assert_array_equal(ri.cpu().numpy(), g["receiver_indices"])
    np.testing.assert_array_equal(rv.cpu().numpy(), g["receiver_valid"])
    assign = mn.dtem_select(3, s, rv)
    np.testing.assert_allclose(assign.cpu().numpy(), g["assign"], rtol=0, atol=2e-6)
    dense = torch.zeros(2, 7, 8, dtype=torch.float32)
    dense.scatter_add_(2, ri.cpu(), assign.cpu() * rv.cpu())
    np.testing.assert_allclose(dense.numpy(), g["dense_assign"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_sparse_score_dtypes(dev, dtype):
    import mergenet_b200 as mn
    grid = (6, 8)
    nbr, val = mn.build_patch_spatial_neighbors(grid, 3.0, device=dev)
    gen = torch.Generator().manual_seed(5)
    perm = torch.stack([torch.randperm(48, generator=gen) for _ in range(3)])
    ai = perm[:, :24].sort(1).values
    bi = perm[:, 24:].sort(1).values
    a = torch.randn(3, 24, 64, generator=gen).to(dtype)
    b = torch.randn(3, 24, 64, generator=gen).to(dtype)
    s, ri, rv = mn.sparse_spatial_score(a.to(dev), b.to(dev), nbr, val, ai.to(dev), bi.to(dev))
    geom = O.Geometry(grid, 3.0)
    es, eri, erv = O.sparse_spatial_score(a.float().numpy(), b.float().numpy(), geom.nbr_idx, geom.nbr_valid,
                                          ai.numpy(), bi.numpy())
    np.testing.assert_array_equal(ri.cpu().numpy(), eri)
    np.testing.assert_array_equal(rv.cpu().numpy(), erv)
    tol = 5e-2 if dtype != torch.float32 else 5e-5
    np.testing.assert_allclose(s.float().cpu().numpy(), es, rtol=tol, atol=tol)
    d = mn.sparse_neighbor_dot(a.to(dev), b.to(dev), ri, rv)
    np.testing.assert_allclose(d.float().cpu().numpy(), es, rtol=tol, atol=tol)


def test_sparse_transport_matches_reference(dev, golden_dir):
    import mergenet_b200 as mn
    g = np.load(golden_dir / "transport.npz")
    args = [torch.from_numpy(g[k]).to(dev) for k in ("assignment", "values", "receiver_indices", "receiver_valid")]
    out = mn.sparse_weighted_transport(*args, int(g["receivers"]))
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("dtype,channels", [(torch.float32, 1), (torch.float32, 32), (torch.float16, 32),
                                            (torch.bfloat16, 384)])
def test_sparse_transport_pair_and_adjoint(dev, dtype, channels):
    """Large-batch transport (tests/test_dtem_spatial_sparse.py:466-498) and
    its adjoint against autograd of the dense scatter."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(20260924)
    batch, donors, receivers, neighbors = 32, 11, 13, 7
    idx = torch.randint(receivers, (batch, donors, neighbors), generator=gen)
    valid = torch.rand(batch, donors, neighbors, generator=gen) > 0.2
    w = torch.rand(batch, donors, neighbors, generator=gen)
    v = torch.randn(batch, donors, channels, generator=gen)
    m = torch.rand(batch, donors, generator=gen)
    feats, mass = mn.sparse_weighted_transport_pair(w.to(dtype).to(dev), v.to(dtype).to(dev), m.to(dtype).to(dev),
                                                    idx.to(dev), valid.to(dev), receivers)
    exp_f = O.sparse_weighted_transport(w.to(dtype).float().numpy(), v.to(dtype).float().numpy(), idx.numpy(),
                                        valid.numpy(), receivers)
    exp_m = O.sparse_weighted_transport(w.to(dtype).float().numpy(), m.to(dtype).float().numpy()[..., None],
                                        idx.numpy(), valid.numpy(), receivers)[..., 0]
    tol = 2e-2 if dtype != torch.float32 else 1e-5
    np.testing.assert_allclose(feats.float().cpu().numpy(), exp_f, rtol=tol, atol=tol)
    np.testing.assert_allclose(mass.float().cpu().numpy(), exp_m, rtol=tol, atol=tol)
    # adjoint
    wg = w.double().requires_grad_()
    vg = v.double().requires_grad_()
    dense = torch.zeros(batch, receivers, channels, dtype=torch.float64)
    dense = dense.scatter_add(1, idx.flatten(1).unsqueeze(-1).expand(-1, -1, channels),
                              (wg.unsqueeze(-1) * vg.unsqueeze(2) * valid.unsqueeze(-1)).flatten(1, 2))
    probe = torch.randn(batch, receivers, channels, generator=gen, dtype=torch.float64)
    gw_ref, gv_ref = torch.autograd.grad((dense * probe).sum(), (wg, vg))
    gw, gv = mn.sparse_transport_adjoint(w.to(dtype).to(dev), v.to(dtype).to(dev), idx.to(dev), valid.to(dev),
                                         probe.to(dtype).to(dev))
    tol = 5e-2 if dtype != torch.float32 else 1e-4
    np.testing.assert_allclose(gw.float().cpu().numpy(), gw_ref.numpy(), rtol=tol, atol=tol * max(1, channels ** 0.5))
    np.testing.assert_allclose(gv.float().cpu().numpy(), gv_ref.numpy(), rtol=tol, atol=tol)
    assert int(torch.count_nonzero(gw.cpu()[~valid])) == 0
    # autograd through sparse_weighted_transport runs the same adjoint
    wd = w.to(dtype).to(dev).requires_grad_()
    vd = v.to(dtype).to(dev).requires_grad_()
    mn.sparse_weighted_transport(wd, vd, idx.to(dev), valid.to(dev), receivers).backward(probe.to(dtype).to(dev))
    assert torch.equal(wd.grad, gw) and torch.equal(vd.grad, gv)


def test_thre_topk_matches_reference(dev, golden_dir):
    import mergenet_b200 as mn
    g = np.load(golden_dir / "thre_topk.npz")
    for i in range(4):
        y = mn.ThreTopK(torch.from_numpy(g[f"x{i}"]).to(dev), int(g[f"k{i}"]), 30.0)
        np.testing.assert_allclose(y.cpu().numpy().reshape(g[f"y{i}"].shape), g[f"y{i}"], rtol=0, atol=2e-6)


def test_thre_topk_backward_matches_reference(dev, golden_dir):
    """x.grad through mn.ThreTopK against the reference's own autograd
    (thetopk.py:4-43), tied rows included (their bracket side follows the
    stable sort; the range gradient is split over tied maxima / minima)."""
    import mergenet_b200 as mn
    g = np.load(golden_dir / "thre_topk_backward.npz")
    for i in range(int(g["count"])):
        x = torch.from_numpy(g[f"x{i}"]).to(dev).requires_grad_(True)
        y = mn.ThreTopK(x, int(g[f"k{i}"]), 30.0)
        np.testing.assert_allclose(y.detach().cpu().numpy(), g[f"y{i}"], rtol=0, atol=2e-6)
        y.backward(torch.from_numpy(g[f"g{i}"]).to(dev))
        ref = g[f"dx{i}"]
        err = np.abs(x.grad.cpu().numpy() - ref).max()
        assert err <= 1e-4 * np.abs(ref).max(), (i, err)


@pytest.mark.parametrize("rows,n,k", [(64, 392, 196), (8, 1000, 37), (3, 4096, 2048)])
def test_thre_topk_backward_large_rows(dev, rows, n, k):
    """Row lengths of the donor sets and the kernel's maximum against the
    float64 closed form of the oracle (rel. 1e-4 of the largest entry)."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(rows * 7 + n)
    x = torch.randn(rows, n, generator=gen) * 3 + 1
    gy = torch.randn(rows, n, generator=gen)
    ref = O.thre_topk_backward(x.numpy(), k, gy.numpy())
    gx = mn.thre_topk_backward(x.to(dev), k, gy.to(dev))
    err = np.abs(gx.cpu().numpy() - ref).max()
    assert err <= 1e-4 * np.abs(ref).max(), err


def test_select_infeasible_budget_fails_closed(dev):
    import mergenet_b200 as mn
    scores = torch.randn(1, 2, 3, device=dev)
    allowed = torch.zeros(1, 2, 3, dtype=torch.bool, device=dev)
    with pytest.raises(RuntimeError):
        mn.dtem_select(1, scores, allowed)


def test_select_degenerate_range_fails_closed(dev):
    """Equal scores everywhere give every donor row the same energy, so the
    ThreTopK range (global max - min, thetopk.py:12-13) is zero and the
    reference divides by it; the kernel flags MN_STATUS_DEGENERATE_RANGE
    (and only that bit) and the host raises instead of returning NaNs."""
    import mergenet_b200 as mn
    from mergenet_b200 import _lib as L
    scores = torch.full((2, 50, 9), 0.3, device=dev)
    allowed = torch.ones(2, 50, 9, dtype=torch.bool, device=dev)
    with pytest.raises(RuntimeError, match="range"):
        mn.dtem_select(10, scores, allowed)
    s = scores.contiguous()
    out = torch.empty_like(s)
    wsb = L.lib().mn_dtem_select_workspace_bytes(2, 50)
    ws = torch.empty(int(wsb), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L.check(L.lib().mn_dtem_select(2, 50, 9, L.ptr(s), L.ptr(allowed.to(torch.uint8)), 10, 1.0, 30.0, L.ptr(out),
                                   L.ptr(ws), wsb, L.ptr(status), L.stream_of(s)), "mn_dtem_select")
    assert int(status.item()) == L.MN_STATUS_DEGENERATE_RANGE
    # a well-posed call on the same context afterwards is unaffected
    gen = torch.Generator().manual_seed(3)
    good = torch.randn(2, 50, 9, generator=gen)
    got = mn.dtem_select(10, good.to(dev), allowed).cpu().numpy()
    want, _, _ = O.select(10, good.numpy(), np.ones((2, 50, 9), dtype=bool))
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-6)


def test_select_empty_rows_stay_finite(dev):
    """tests/test_dtem_spatial_mask.py:205-239: an isolated donor keeps its mass."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(1)
    scores = torch.randn(2, 6, 5, generator=gen)
    allowed = torch.rand(2, 6, 5, generator=gen) > 0.4
    allowed[:, 0] = False
    assign = mn.dtem_select(2, scores.to(dev), allowed.to(dev)).cpu()
    want, _, _ = O.select(2, scores.numpy(), allowed.numpy())
    assert bool(torch.isfinite(assign).all())
    assert int(torch.count_nonzero(assign[:, 0])) == 0
    assert int(torch.count_nonzero(assign[~allowed])) == 0
    np.testing.assert_allclose(assign.numpy(), want, rtol=0, atol=2e-6)


def test_carrier_scatter_is_gather_transpose(dev):
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(2)
    idx = torch.stack([torch.randperm(20, generator=gen)[:8] for _ in range(3)]).to(dev)
    topk_x = torch.randn(3, 9, 16, generator=gen).to(dev)
    full = mn.carrier_scatter(topk_x, idx, 20)
    back = torch.gather(full, 1, idx.unsqueeze(-1).expand(-1, -1, 16))
    assert torch.equal(back, topk_x[:, 1:])
    mask = torch.ones(3, 20, dtype=torch.bool, device=dev)
    mask.scatter_(1, idx, False)
    assert int(torch.count_nonzero(full[mask])) == 0


@pytest.mark.parametrize("dtype,channels", [(torch.float16, 384), (torch.float32, 13), (torch.bfloat16, 8)])
def test_carrier_scatter_one_pass(dev, dtype, channels):
    """The scatter writes every patch row once: the carrier's features at its
    patch, zeros elsewhere (config-2 shapes: 392 of 784 patches), on the
    16-byte path and the element path; a patch listed twice takes the later
    carrier."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(channels)
    b, p, k = 4, 784, 392
    idx = torch.stack([torch.randperm(p, generator=gen)[:k] for _ in range(b)])
    idx[3, 10] = idx[3, 3]  # patch listed twice: carrier 10 wins over carrier 3
    topk_x = torch.randn(b, k + 1, channels, generator=gen).to(dtype)
    want = torch.zeros(b, p, channels, dtype=dtype)
    for i in range(b):
        for j in range(k):
            want[i, idx[i, j]] = topk_x[i, 1 + j]
    got = mn.carrier_scatter(topk_x.to(dev), idx.to(dev), p)
    assert torch.equal(got.cpu(), want)


def test_empty_batches(dev):
    import mergenet_b200 as mn
    nbr, val = mn.build_patch_spatial_neighbors((3, 5), 2, device=dev)
    a = torch.empty(0, 7, 9, device=dev)
    b = torch.empty(0, 8, 9, device=dev)
    e = torch.empty(0, 7, dtype=torch.long, device=dev)
    s, ri, rv = mn.sparse_spatial_score(a, b, nbr, val, e, torch.empty(0, 8, dtype=torch.long, device=dev))
    assert s.shape == (0, 7, nbr.shape[1])
    out = mn.sparse_weighted_transport(torch.empty(0, 7, nbr.shape[1], device=dev), a, ri, rv, 8)
    assert out.shape == (0, 8, 9)


def test_neighbor_dot_backward_matches_reference(dev, golden_dir):
    """Gradients of sparse_neighbor_dot against the reference's own autograd
    run (_SparseNeighborDot.backward, dtem.py:633-677, torch path): grad_b is
    summed in the reference's edge order, so it matches bit for bit."""
    import mergenet_b200 as mn
    g = np.load(golden_dir / "neighbor_dot_backward.npz")
    for i in range(2):
        a = torch.from_numpy(g[f"a{i}"]).to(dev).requires_grad_(True)
        b = torch.from_numpy(g[f"b{i}"]).to(dev).requires_grad_(True)
        ridx = torch.from_numpy(g[f"receiver_indices{i}"]).to(dev)
        rval = torch.from_numpy(g[f"receiver_valid{i}"]).to(dev)
        scores = mn.sparse_neighbor_dot(a, b, ridx, rval)
        scores.backward(torch.from_numpy(g[f"grad_scores{i}"]).to(dev))
        np.testing.assert_allclose(scores.detach().cpu().numpy(), g[f"scores{i}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(a.grad.cpu().numpy(), g[f"grad_a{i}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_array_equal(b.grad.cpu().numpy(), g[f"grad_b{i}"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_spatial_score_backward(dev, golden_dir, dtype):
    """sparse_spatial_score is differentiable in a and b, with the receiver
    slots it returns (dtem.py:768-810): checked against the oracle's
    neighbor-dot gradients on those slots."""
    import mergenet_b200 as mn
    g = np.load(golden_dir / "select_g3x5.npz")
    nbr, val = mn.build_patch_spatial_neighbors((3, 5), 2, device=dev)
    a = torch.from_numpy(g["a"]).to(dev, dtype).requires_grad_(True)
    b = torch.from_numpy(g["b"]).to(dev, dtype).requires_grad_(True)
    scores, ridx, rval = mn.sparse_spatial_score(a, b, nbr, val, torch.from_numpy(g["a_idx"] - 1).to(dev),
                                                 torch.from_numpy(g["b_idx"] - 1).to(dev))
    assert not ridx.requires_grad and not rval.requires_grad
    gs = torch.randn(scores.shape, generator=torch.Generator().manual_seed(3)).to(dev, dtype)
    scores.backward(gs)
    want_a, want_b = O.sparse_neighbor_dot_backward(g["a"], g["b"], ridx.cpu().numpy(), rval.cpu().numpy(),
                                                    gs.float().cpu().numpy())
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    np.testing.assert_allclose(a.grad.float().cpu().numpy(), want_a, rtol=tol, atol=tol)
    np.testing.assert_allclose(b.grad.float().cpu().numpy(), want_b, rtol=tol, atol=tol)


def test_select_backward_matches_reference(dev, golden_dir):
    """Metric gradients through the sparse score and the soft-k-max select
    against the reference's autograd through DTEMBlock._select
    (dtem.py:1464-1580), and the select block's own score gradient; one case
    has donor rows with no allowed receiver."""
    import mergenet_b200 as mn
    g = np.load(golden_dir / "select_backward.npz")
    for i in range(int(g["count"])):
        nbr, val = mn.build_patch_spatial_neighbors(tuple(int(v) for v in g[f"grid{i}"]), float(g[f"radius{i}"]),
                                                    device=dev)
        a = torch.from_numpy(g[f"a{i}"]).to(dev).requires_grad_(True)
        b = torch.from_numpy(g[f"b{i}"]).to(dev).requires_grad_(True)
        scores, ridx, rval = mn.sparse_spatial_score(a, b, nbr, val, torch.from_numpy(g[f"a_idx{i}"] - 1).to(dev),
                                                     torch.from_numpy(g[f"b_idx{i}"] - 1).to(dev))
        scores.retain_grad()
        assign = mn.dtem_select(int(g[f"k{i}"]), scores, rval)
        np.testing.assert_allclose(assign.detach().cpu().numpy(), g[f"assign{i}"], rtol=0, atol=2e-6)
        assign.backward(torch.from_numpy(g[f"grad_assign{i}"]).to(dev))
        for name, got in (("grad_scores", scores.grad), ("grad_a", a.grad), ("grad_b", b.grad)):
            ref = g[f"{name}{i}"]
            err = np.abs(got.cpu().numpy() - ref).max()
            assert err <= 1e-4 * np.abs(ref).max(), (i, name, err)


@pytest.mark.parametrize("batch,na,k_slots,k", [(4, 392, 29, 196), (2, 1000, 13, 300)])
def test_select_backward_against_oracle(dev, batch, na, k_slots, k):
    """Donor-set sizes of the 28x28 grid (radius 3: 29 slots) and a longer
    row against the oracle's float64 closed form; about a tenth of the slots
    and a few whole rows are masked."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(na + k)
    scores = torch.randn(batch, na, k_slots, generator=gen) * 0.3
    allowed = torch.rand(batch, na, k_slots, generator=gen) > 0.1
    allowed[:, ::97] = False
    ga = torch.randn(batch, na, k_slots, generator=gen)
    ref = O.select_backward(k, scores.numpy(), allowed.numpy(), ga.numpy())
    got = mn.dtem_select_backward(k, scores.to(dev), allowed.to(dev), ga.to(dev))
    err = np.abs(got.cpu().numpy() - ref).max()
    assert err <= 1e-4 * np.abs(ref).max(), err
    assert int(torch.count_nonzero(got.cpu()[~allowed])) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_precision_gradients_follow_the_input_dtype(dev, dtype):
    """Autocast-style 16-bit inputs: ThreTopK and the select compute in fp32
    (as the reference's float32 energies and scores do) and hand back
    gradients in the input's dtype, equal to the fp32 gradients rounded."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(21)
    x = (torch.randn(6, 392, generator=gen) * 2 + 4).to(dtype)
    gy = torch.randn(6, 392, generator=gen)
    xh = x.to(dev).requires_grad_(True)
    mn.ThreTopK(xh, 196).backward(gy.to(dev).to(dtype))
    want = mn.thre_topk_backward(x.float().to(dev), 196, gy.to(dtype).float().to(dev))
    assert xh.grad.dtype == dtype
    torch.testing.assert_close(xh.grad, want.to(dtype), rtol=0, atol=0)
    scores = (torch.randn(2, 300, 13, generator=gen) * 0.3).to(dtype)
    allowed = torch.rand(2, 300, 13, generator=gen) > 0.1
    ga = torch.randn(2, 300, 13, generator=gen)
    sh = scores.to(dev).requires_grad_(True)
    assign = mn.dtem_select(100, sh, allowed.to(dev))
    assert assign.dtype == dtype
    assign.backward(ga.to(dev).to(dtype))
    want = mn.dtem_select_backward(100, scores.float().to(dev), allowed.to(dev), ga.to(dtype).float().to(dev))
    assert sh.grad.dtype == dtype
    torch.testing.assert_close(sh.grad, want.to(dtype), rtol=0, atol=0)


@pytest.mark.parametrize("channels", [1, 8, 40, 384])
def test_transport_at_the_48x48_grid_size(dev, channels):
    """The drop-in transport at the 384x384 / patch-8 size (1,152 donors and
    receivers, 29 slots): its edge list and sort counts fit the shared
    memory, and every (receiver, channel) sum is the oracle's sequential
    donor-major scatter, bit for bit, on the narrow (thread per receiver)
    and wide (four channels per lane) paths."""
    import mergenet_b200 as mn
    gen = torch.Generator().manual_seed(48 + channels)
    b, na, nb, k = 2, 1152, 1152, 29
    w = torch.rand(b, na, k, generator=gen)
    v = torch.randn(b, na, channels, generator=gen)
    ridx = torch.randint(nb, (b, na, k), generator=gen)
    rvalid = torch.rand(b, na, k, generator=gen) > 0.4
    got = mn.sparse_weighted_transport(w.to(dev), v.to(dev), ridx.to(dev), rvalid.to(dev), nb)
    want = O.sparse_weighted_transport(w.numpy(), v.numpy(), ridx.numpy(), rvalid.numpy(), nb)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
