"""The module-level drop-ins driven the way the reference's callers drive them.

DTEMMergeBlock runs the reference's merge loop (LocalEncoder.forward,
opentome/models/mergenet/model.py:574-590) and carrier block (:1157-1183) on
CUDA tensors, and is checked against the fixtures make_golden.py recorded
from the reference's own DTEMBlock._merge_train / _select: per layer the
assignment and the ``_tome_info`` side effects (assign_layout,
assign_b_indices, assign_valid_mask), then the masses, token_center and the
carriers.
"""
import numpy as np
import pytest
import torch

from conftest import carrier_mismatches, rel_err
from inputs import canonical_r_list, routing_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import mergenet_b200  # noqa: F401
    return torch.device("cuda", 0)


def run_reference_loop(block, x, metrics, r_list):
    """make_golden.run_routing's loop, on the drop-in block: the six
    _merge_train calls with merge_layer_index set per layer, recording what
    _select leaves in _tome_info, then the carrier block's tensor ops."""
    layers = []
    original = block._select

    def recording_select(k, a, b, a_orig_idx=None, b_orig_idx=None):
        assign, out = original(k, a, b, a_orig_idx, b_orig_idx)
        info = block._tome_info
        layers.append(dict(layout=info["assign_layout"], assign=assign.cpu().numpy(),
                           receiver_indices=info["assign_b_indices"].cpu().numpy(),
                           receiver_valid=info["assign_valid_mask"].cpu().numpy()))
        return assign, out

    block._select = recording_select
    bsz, t, _ = x.shape
    size = torch.ones(bsz, t, 1, device=x.device)
    n = t
    for i, r in enumerate(r_list):
        block._tome_info["merge_layer_index"] = i
        x, size, n, _, _ = block._merge_train(x, size, r, n, {"metric": metrics[i]})
    center = block._tome_info["token_center"]
    k = t - sum(r_list) - 1
    strength = size[..., 0][:, 1:]
    _, topk_indices = torch.topk(strength, k, dim=1, largest=True, sorted=False)
    order = torch.argsort(torch.gather(center[:, 1:], 1, topk_indices), dim=1)
    topk = torch.gather(topk_indices, 1, order)
    topk_x = torch.cat([x[:, :1], torch.gather(x, 1, (topk + 1).unsqueeze(-1).expand(-1, -1, x.shape[-1]))], 1)
    return layers, size[..., 0], center, topk, topk_x


@pytest.mark.parametrize("name", ["route_c1", "route_g3x6", "route_g4x4"])
def test_merge_block_through_the_reference_loop(dev, golden_dir, name):
    import mergenet_b200 as mn
    g = np.load(golden_dir / f"{name}.npz")
    grid = tuple(int(v) for v in g["grid"])
    r_list = [int(v) for v in g["r_list"]]
    x, metrics = routing_inputs(int(g["seed"]), int(g["batch"]), grid, int(g["channels"]), int(g["metric_dim"]),
                                layers=len(r_list))
    block = mn.make_merge_block(grid, float(g["radius"]), device=dev)
    layers, size, center, topk, topk_x = run_reference_loop(
        block, torch.from_numpy(x).to(dev), torch.from_numpy(metrics).to(dev), r_list)
    assert len(layers) == len(r_list)
    for i, layer in enumerate(layers):
        assert layer["layout"] == "spatial_sparse"
        if f"assign_{i}" in g:
            np.testing.assert_array_equal(layer["receiver_indices"], g[f"receiver_indices_{i}"])
            np.testing.assert_array_equal(layer["receiver_valid"], g[f"receiver_valid_{i}"])
            np.testing.assert_allclose(layer["assign"], g[f"assign_{i}"], rtol=0, atol=5e-6)
    np.testing.assert_allclose(size.cpu().numpy(), g["size"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(center.cpu().numpy(), g["center"], rtol=0, atol=2e-3)
    mism = carrier_mismatches(topk.cpu().numpy(), g["topk_idx"], g["center"])
    assert not mism, mism
    if "topk_x" in g:
        assert rel_err(topk_x.cpu().numpy(), g["topk_x"]) <= 2e-3


def test_merge_block_matches_fused_route(dev):
    """The function-level path (six DTEMMergeBlock layers) and the fused
    RoutePlan give the same carriers, masses and centres on one input."""
    import mergenet_b200 as mn
    from inputs import canonical_r_list
    grid = (28, 28)
    r_list = canonical_r_list(grid)
    x, metrics = routing_inputs(11, 3, grid, 64, 64)
    xt, mt = torch.from_numpy(x).to(dev), torch.from_numpy(metrics).to(dev)
    block = mn.make_merge_block(grid, 3.0, device=dev)
    _, size, center, topk, topk_x = run_reference_loop(block, xt, mt, r_list)
    res = mn.RoutePlan(grid, 3.0, r_list, device=dev)(xt, mt)
    mism = carrier_mismatches(res.topk_idx.cpu().numpy(), topk.cpu().numpy(), center.cpu().numpy())
    assert not mism, mism
    torch.testing.assert_close(res.size, size, rtol=3e-5, atol=3e-5)
    torch.testing.assert_close(res.center, center, rtol=0, atol=2e-3)
    assert rel_err(res.topk_x.cpu().numpy(), topk_x.cpu().numpy()) <= 2e-3


@pytest.mark.parametrize("dtype,cls_global", [(torch.float16, True), (torch.bfloat16, False)])
def test_local_attention_module(dev, dtype, cls_global):
    """LocalAttention (bias_local_attn.py:633-724) with the reference's
    parameter names, against its forward restated in PyTorch: qkv Linear,
    band-masked softmax over |i - j| <= 16 in fp32, CLS row over every key,
    proj Linear."""
    import math
    import mergenet_b200 as mn
    torch.manual_seed(3)
    mod = mn.LocalAttention(384, num_heads=6, qkv_bias=True, local_window=16, cls_global=cls_global).to(dev, dtype)
    x = torch.randn(2, 785, 384, device=dev, dtype=dtype)
    with torch.no_grad():
        out = mod(x)
        qkv = mod.qkv(x).view(2, 785, 3, 6, 64).permute(2, 0, 3, 1, 4).float()
        q, k, v = qkv.unbind(0)
        s = q @ k.transpose(-1, -2) / math.sqrt(64)
        pos = torch.arange(785, device=dev)
        band = (pos[:, None] - pos[None, :]).abs() <= 16
        if cls_global:
            band[0] = True
        a = torch.softmax(s.masked_fill(~band, float("-inf")), -1) @ v
        want = mod.proj(a.transpose(1, 2).reshape(2, 785, 384).to(dtype)).float()
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-2
    assert ((out.float() - want).abs().max() / want.abs().max()).item() <= tol
    assert sorted(n for n, _ in mod.named_parameters()) == ["proj.bias", "proj.weight", "qkv.bias", "qkv.weight"]


@pytest.mark.parametrize("case", [0, 1])
def test_merge_block_training_gradients_match_reference(dev, golden_dir, case):
    """A training-mode merge layer (dtem.py:1687-2223) forward and backward
    against the reference's own autograd: output tokens, masses and centres,
    then the gradients with respect to x, size and the metric, which run
    through the transport adjoint, the select backward (ThreTopK included)
    and the neighbour-dot backward, and the straight-through mass update."""
    import mergenet_b200 as mn
    g = np.load(golden_dir / "merge_train_backward.npz")
    i = case
    grid = tuple(int(v) for v in g[f"grid{i}"])
    block = mn.make_merge_block(grid, float(g[f"radius{i}"]), device=dev).train()
    block._tome_info.update({"train_grouping": str(g[f"grouping{i}"]), "train_grouping_seed": 7,
                             "merge_layer_index": int(g[f"layer{i}"])})
    x = torch.from_numpy(g[f"x{i}"]).to(dev).requires_grad_(True)
    metric = torch.from_numpy(g[f"metric{i}"]).to(dev).requires_grad_(True)
    size = torch.from_numpy(g[f"size{i}"]).to(dev).requires_grad_(True)
    t = x.shape[1]
    x_out, size_out, n, _, _ = block._merge_train(x, size, int(g[f"r{i}"]), t, {"metric": metric})
    assert n == t
    np.testing.assert_allclose(x_out.detach().cpu().numpy(), g[f"x_out{i}"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(size_out.detach().cpu().numpy(), g[f"size_out{i}"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(block._tome_info["token_center"].cpu().numpy(), g[f"center{i}"], rtol=0, atol=1e-3)
    torch.autograd.backward([x_out, size_out], [torch.from_numpy(g[f"grad_x_out{i}"]).to(dev),
                                                torch.from_numpy(g[f"grad_size_out{i}"]).to(dev)])
    for name, got in (("grad_x", x.grad), ("grad_size", size.grad), ("grad_metric", metric.grad)):
        ref = g[f"{name}{i}"]
        err = np.abs(got.cpu().numpy() - ref).max()
        assert err <= 1e-4 * np.abs(ref).max(), (name, err)


def test_merge_block_training_random_groups(dev):
    """The default train grouping ("random_per_sample", dtem.py:1763-1770):
    each image gets its own donor / receiver split from torch.rand on the
    device, mass is conserved, the same generator state gives the same
    layer, and the backward reaches x, size and the metric."""
    import mergenet_b200 as mn
    grid = (14, 14)
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(4, 197, 32, generator=gen).to(dev).requires_grad_(True)
    metric = torch.randn(4, 197, 16, generator=gen).to(dev).requires_grad_(True)
    size = torch.ones(4, 197, 1, device=dev, requires_grad=True)
    outs = []
    for _ in range(2):
        block = mn.make_merge_block(grid, 3.0, device=dev).train()
        torch.cuda.manual_seed(1234)
        outs.append(block._merge_train(x, size, 40, 197, {"metric": metric}))
    (x0, s0, _, _, _), (x1, s1, _, _, _) = outs
    assert torch.equal(x0, x1) and torch.equal(s0, s1)
    torch.testing.assert_close(s0.double().sum(1), size.double().sum(1), rtol=1e-6, atol=1e-4)
    # different images, different splits: the tokens that gave mass away
    # (donors, mass now below 1) sit at different positions
    gave = (s0[..., 0] < 1).cpu()
    assert int(gave[:, 1:].sum(1).min()) > 0
    assert any(not torch.equal(gave[0], gave[j]) for j in range(1, 4))
    (x0 * torch.randn_like(x0)).sum().add((s0 * 0.5).sum()).backward()
    for t in (x, size, metric):
        assert t.grad is not None and bool(torch.isfinite(t.grad).all())
    assert float(metric.grad.abs().sum()) > 0


def test_merge_chain_training_gradients_match_reference(dev, golden_dir):
    """Six training-mode merge layers chained as LocalEncoder.forward chains
    them (model.py:574-590), then the carrier top-k and gather
    (model.py:1157-1183), against the reference's own autograd of the same
    chain: outputs, carriers, centres, and the gradients with respect to the
    input tokens and all six metrics."""
    import mergenet_b200 as mn
    g = np.load(golden_dir / "merge_train_chain_backward.npz")
    grid = tuple(int(v) for v in g["grid"])
    r_list = [int(v) for v in g["r_list"]]
    block = mn.make_merge_block(grid, float(g["radius"]), device=dev).train()
    block._tome_info.update({"train_grouping": "alternating_per_layer_fast", "train_grouping_seed": 0})
    x = torch.from_numpy(g["x"]).to(dev).requires_grad_(True)
    metrics = torch.from_numpy(g["metrics"]).to(dev).requires_grad_(True)
    bsz, t, c = x.shape
    xs, size, n = x, torch.ones(bsz, t, 1, device=dev), t
    for i, r in enumerate(r_list):
        block._tome_info["merge_layer_index"] = i
        xs, size, n, _, _ = block._merge_train(xs, size, r, n, {"metric": metrics[i]})
    k = t - sum(r_list) - 1
    idx = torch.topk(size[..., 0][:, 1:].detach(), k, dim=1, largest=True, sorted=False).indices
    order = torch.argsort(torch.gather(block._tome_info["token_center"][:, 1:], 1, idx), dim=1)
    topk = torch.gather(idx, 1, order)
    np.testing.assert_array_equal(topk.cpu().numpy(), g["topk_idx"])
    carriers = torch.gather(xs, 1, (topk + 1).unsqueeze(-1).expand(-1, -1, c))
    np.testing.assert_allclose(xs.detach().cpu().numpy(), g["x_out"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(size.detach().cpu().numpy(), g["size_out"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(block._tome_info["token_center"].cpu().numpy(), g["center"], rtol=0, atol=2e-3)
    torch.autograd.backward([xs, size, carriers], [torch.from_numpy(g[k_]).to(dev) for k_ in
                                                   ("grad_x_out", "grad_size_out", "grad_carriers")])
    for name, got in (("grad_x", x.grad), ("grad_metrics", metrics.grad)):
        ref = g[name]
        err = np.abs(got.cpu().numpy() - ref).max()
        assert err <= 1e-3 * np.abs(ref).max(), (name, err)


def test_merge_block_loop_at_the_48x48_grid(dev):
    """The drop-in merge block driven through the six-layer loop at the
    384x384 / patch-8 size (2,305 tokens, radius 3) gives the fused route's
    carriers, masses and centres on the same inputs."""
    import mergenet_b200 as mn
    grid = (48, 48)
    r_list = canonical_r_list(grid)
    x, metrics = routing_inputs(17, 2, grid, 24, 64, layers=6, metric_dtype=np.float32)
    xt, mt = torch.from_numpy(x).to(dev), torch.from_numpy(metrics).to(dev)
    block = mn.make_merge_block(grid, 3.0, device=dev)
    _, size, center, topk, topk_x = run_reference_loop(block, xt, mt, r_list)
    res = mn.RoutePlan(grid, 3.0, r_list, device=dev)(xt, mt)
    mism = carrier_mismatches(topk.cpu().numpy(), res.topk_idx.cpu().numpy(), res.center.cpu().numpy())
    assert not mism, mism
    np.testing.assert_allclose(size.cpu().numpy(), res.size.cpu().numpy(), rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(center.cpu().numpy(), res.center.cpu().numpy(), rtol=0, atol=2e-3)
    assert rel_err(topk_x.cpu().numpy(), res.topk_x.cpu().numpy()) <= 2e-3
