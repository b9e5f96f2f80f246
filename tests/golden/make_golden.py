#!/usr/bin/env python3
"""Generate golden fixtures by running the MergeNet reference itself.

Run where a checkout of the reference is available (read-only), naming it
in $MERGENET_REFERENCE:

    MERGENET_REFERENCE=<path to the MergeNet checkout> python tests/golden/make_golden.py

The reference's routing modules import timm at module level; timm is not
installed, so ``timm_shim/`` (inert placeholders written for this repository)
satisfies those imports.  Everything computed here runs the reference's own
code: ``DTEMBlock._merge_train`` / ``_select`` (opentome/timm/dtem.py),
``sparse_spatial_score`` / ``sparse_weighted_transport`` and ``ThreTopK``
(opentome/utils/thetopk.py).  The carrier block of
``CLSHybridToMeModel.forward`` (opentome/models/mergenet/model.py:1157-1183)
needs the full timm model, so its five tensor ops (topk, gather, argsort,
gather, gather) are executed here in the same order on the reference's
outputs.  Inputs come from ``inputs.py`` and are regenerated from their seed
by the tests; only outputs are stored.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if "MERGENET_REFERENCE" not in os.environ:
    raise SystemExit("set MERGENET_REFERENCE to the MergeNet reference checkout")
REF = Path(os.environ["MERGENET_REFERENCE"])
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE / "timm_shim"))
sys.path.insert(0, str(REF))

import torch  # noqa: E402

from inputs import canonical_r_list, routing_inputs  # noqa: E402
from opentome.timm.dtem import (  # noqa: E402
    DTEMBlock,
    adjacency_to_padded_neighbors,
    build_patch_spatial_adjacency,
    sparse_neighbor_dot,
    sparse_spatial_score,
    sparse_weighted_transport,
)
from opentome.utils.thetopk import ThreTopK  # noqa: E402
from opentome.timm.bias_local_attn import (  # noqa: E402
    naive_biased_local_attention,
    naive_unbiased_local_attention,
)

torch.set_num_threads(max(1, os.cpu_count() or 1))


def make_block(grid, radius, backend):
    """Bare DTEMBlock with a hand-filled _tome_info, as the reference's own
    tests build it (tests/test_dtem_spatial_sparse.py:27-47, :281-304)."""
    adjacency = build_patch_spatial_adjacency(grid, radius)
    nbr, valid = adjacency_to_padded_neighbors(adjacency)
    block = DTEMBlock.__new__(DTEMBlock)
    torch.nn.Module.__init__(block)
    block._tome_info = {
        "window_size": 0,
        "dtem_spatial_radius": radius,
        "dtem_spatial_metric": "euclidean",
        "dtem_spatial_backend": backend,
        "patch_grid_size": grid,
        "num_prefix_tokens": 1,
        "spatial_adjacency": adjacency,
        "spatial_neighbor_indices": nbr,
        "spatial_neighbor_valid": valid,
        "tau1": 1.0,
        "tau2": 30.0,
        "use_softkmax": True,
        "collect_merge_stats": False,
        "class_token": True,
        "distill_token": False,
        "source_trace_mode": "center",
        "trace_source": False,
        "source_tracking_mode": "none",
        "local_depth": 6,
        "eval_grouping": "alternating_per_layer_fast",
        "eval_grouping_seed": 0,
        "merge_layer_index": 0,
        "t": 1,
        "token_center": None,
    }
    block.eval()
    return block


def run_routing(x, metrics, r_list, grid, radius, backend="sparse", capture=False):
    """Reference merge loop (model.py:574-590) + carrier block (:1157-1183)."""
    block = make_block(grid, radius, backend)
    layers = []
    if capture:
        original = DTEMBlock._select

        def recording_select(k, a, b, a_orig_idx=None, b_orig_idx=None):
            assign, out = original(block, k, a, b, a_orig_idx, b_orig_idx)
            layers.append(dict(
                assign=assign.detach().numpy().copy(),
                receiver_indices=block._tome_info["assign_b_indices"].numpy().copy(),
                receiver_valid=block._tome_info["assign_valid_mask"].numpy().copy()))
            return assign, out

        block._select = recording_select
    bsz, t, _ = x.shape
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    size = torch.ones(bsz, t, 1)
    n = t
    with torch.no_grad():
        for i, r in enumerate(r_list):
            block._tome_info["merge_layer_index"] = i
            # fp16 autocast computes the metric norm in fp32 and promotes the
            # division to fp32; on the CPU reproduce that by upcasting first.
            m = torch.from_numpy(np.ascontiguousarray(metrics[i]).astype(np.float32))
            xt, size, n, _, _ = block._merge_train(xt, size, r, n, {"metric": m})
        center = block._tome_info["token_center"].float()
        k = t - sum(r_list) - 1
        strength = size[..., 0][:, 1:]
        _, topk_indices = torch.topk(strength, k, dim=1, largest=True, sorted=False)
        topk_com = torch.gather(center[:, 1:], 1, topk_indices)
        sorted_order = torch.argsort(topk_com, dim=1)
        sorted_topk = torch.gather(topk_indices, 1, sorted_order)
        full = sorted_topk + 1
        topk_x = torch.cat([xt[:, :1], torch.gather(xt, 1, full.unsqueeze(-1).expand(-1, -1, xt.shape[-1]))], 1)
        topk_size = torch.cat([size[:, :1, 0], torch.gather(size[..., 0], 1, full)], 1)
    s = np.sort(size[:, 1:, 0].numpy().astype(np.float64), axis=1)[:, ::-1]
    margin = (s[:, k - 1] - s[:, k]) / np.abs(s[:, k - 1])
    out = dict(topk_idx=sorted_topk.numpy().astype(np.int32), size=size[..., 0].numpy(),
               center=center.numpy(), topk_size=topk_size.numpy(), margin=margin)
    return out, topk_x.numpy(), layers


def route_case(name, seed, batch, grid, radius, channels, metric_dim, r_list,
               keep_features=True, capture=False, dense_check=False):
    x, metrics = routing_inputs(seed, batch, grid, channels, metric_dim, layers=len(r_list))
    out, topk_x, layers = run_routing(x, metrics, r_list, grid, radius, capture=capture)
    payload = dict(seed=seed, batch=batch, grid=np.array(grid), radius=radius,
                   channels=channels, metric_dim=metric_dim, r_list=np.array(r_list), **out)
    if keep_features:
        payload["topk_x"] = topk_x
    for i, layer in enumerate(layers):
        payload[f"assign_{i}"] = layer["assign"]
        payload[f"receiver_indices_{i}"] = layer["receiver_indices"].astype(np.int32)
        payload[f"receiver_valid_{i}"] = layer["receiver_valid"]
    if dense_check:
        dense, _, _ = run_routing(x, metrics, r_list, grid, radius, backend="dense")
        payload["dense_topk_idx"] = dense["topk_idx"]
        payload["dense_size"] = dense["size"]
    np.savez_compressed(HERE / f"{name}.npz", **payload)
    print(name, "min margin", float(out["margin"].min()))


def thre_topk_case():
    rng = np.random.default_rng(7)
    cases = {}
    x = (rng.random((4, 37), dtype=np.float32) * 20 + 1).astype(np.float32)
    cases["x0"], cases["k0"] = x, 9
    cases["y0"] = ThreTopK(torch.from_numpy(x), 9, 30.0).numpy()
    x1 = x.copy()
    x1[1, ::3] = 0.0  # invalid rows contribute zero energy to the global range
    cases["x1"], cases["k1"] = x1, 5
    cases["y1"] = ThreTopK(torch.from_numpy(x1), 5, 30.0).numpy()
    x2 = (rng.random(50, dtype=np.float32) * 3).astype(np.float32)
    cases["x2"], cases["k2"] = x2, 20
    cases["y2"] = ThreTopK(torch.from_numpy(x2), 20, 30.0).numpy()
    x3 = (rng.standard_normal((2, 392), dtype=np.float32) * 2 + 12).astype(np.float32)
    cases["x3"], cases["k3"] = x3, 65
    cases["y3"] = ThreTopK(torch.from_numpy(x3), 65, 30.0).numpy()
    np.savez_compressed(HERE / "thre_topk.npz", **cases)


def thre_topk_backward_case():
    """Gradients of the reference's ThreTopK through its own autograd
    (sort, logcumsumexp, the bracket gather and the global max - min range,
    opentome/utils/thetopk.py:4-43) for random upstream gradients."""
    rng = np.random.default_rng(17)
    cases = {}
    shapes = [((4, 37), 9), ((3, 64), 20), ((2, 392), 65), ((1, 50), 49), ((5, 8), 1)]
    for i, (shape, k) in enumerate(shapes):
        x = (rng.standard_normal(shape, dtype=np.float32) * 2 + 5).astype(np.float32)
        g = rng.standard_normal(shape, dtype=np.float32)
        tx = torch.from_numpy(x).requires_grad_(True)
        y = ThreTopK(tx, k, 30.0)
        y.backward(torch.from_numpy(g))
        cases.update({f"x{i}": x, f"k{i}": k, f"g{i}": g, f"y{i}": y.detach().numpy(), f"dx{i}": tx.grad.numpy()})
    # integer-valued rows: ties everywhere, at the bracket and at the global
    # maximum and minimum
    for i, (shape, k) in enumerate([((3, 40), 10), ((2, 64), 31)], start=len(shapes)):
        x = np.round(rng.standard_normal(shape, dtype=np.float32) * 2 + 5).astype(np.float32)
        g = rng.standard_normal(shape, dtype=np.float32)
        tx = torch.from_numpy(x).requires_grad_(True)
        y = ThreTopK(tx, k, 30.0)
        y.backward(torch.from_numpy(g))
        cases.update({f"x{i}": x, f"k{i}": k, f"g{i}": g, f"y{i}": y.detach().numpy(), f"dx{i}": tx.grad.numpy()})
    cases["count"] = np.int64(len(shapes) + 2)
    np.savez_compressed(HERE / "thre_topk_backward.npz", **cases)


def select_case():
    """The reference test's (3,5) R=2 geometry with per-sample partitions
    (tests/test_dtem_spatial_sparse.py:179-227)."""
    grid, radius = (3, 5), 2
    a_idx = torch.tensor([[1, 3, 5, 7, 9, 11, 13], [2, 4, 6, 8, 10, 12, 14]])
    b_idx = torch.tensor([[2, 4, 6, 8, 10, 12, 14, 15], [1, 3, 5, 7, 9, 11, 13, 15]])
    rng = np.random.default_rng(20260820)
    a = rng.standard_normal((2, 7, 9), dtype=np.float32)
    b = rng.standard_normal((2, 8, 9), dtype=np.float32)
    block = make_block(grid, radius, "sparse")
    with torch.no_grad():
        scores, ridx, rvalid = sparse_spatial_score(
            torch.from_numpy(a), torch.from_numpy(b),
            block._tome_info["spatial_neighbor_indices"],
            block._tome_info["spatial_neighbor_valid"], a_idx - 1, b_idx - 1)
        assign, _ = block._select(3, torch.from_numpy(a), torch.from_numpy(b), a_idx, b_idx)
        dense = make_block(grid, radius, "dense")
        dense_assign, _ = dense._select(3, torch.from_numpy(a), torch.from_numpy(b), a_idx, b_idx)
    np.savez_compressed(
        HERE / "select_g3x5.npz", a=a, b=b, a_idx=a_idx.numpy(), b_idx=b_idx.numpy(),
        scores=scores.numpy(), receiver_indices=ridx.numpy().astype(np.int32),
        receiver_valid=rvalid.numpy(), assign=assign.numpy(), dense_assign=dense_assign.numpy())


def transport_case():
    """Random edge lists as in tests/test_dtem_spatial_sparse.py:127-159."""
    rng = np.random.default_rng(20260820)
    batch, donors, receivers, neighbors, channels = 2, 7, 8, 6, 11
    assignment = rng.random((batch, donors, neighbors), dtype=np.float32)
    values = rng.standard_normal((batch, donors, channels), dtype=np.float32)
    ridx = rng.integers(0, receivers, (batch, donors, neighbors))
    rvalid = rng.random((batch, donors, neighbors)) > 0.25
    with torch.no_grad():
        out = sparse_weighted_transport(torch.from_numpy(assignment), torch.from_numpy(values),
                                        torch.from_numpy(ridx), torch.from_numpy(rvalid), receivers)
    np.savez_compressed(HERE / "transport.npz", assignment=assignment, values=values,
                        receiver_indices=ridx.astype(np.int32), receiver_valid=rvalid,
                        receivers=receivers, out=out.numpy())


def select_backward_case():
    """Gradients through the reference's sparse soft-k-max select,
    DTEMBlock._select (opentome/timm/dtem.py:1464-1580): sparse scores,
    masked logsumexp row energies, ThreTopK over the batch, the row softmax
    and the (detached) over-unity renormalisation.  The scores' own gradient
    is observed by wrapping the module's sparse_spatial_score (the call
    itself is the reference's, unchanged) so the select block can be checked
    apart from the score's backward."""
    import opentome.timm.dtem as ref_dtem
    rng = np.random.default_rng(20261203)
    cases = {}
    seen = {}
    original = ref_dtem.sparse_spatial_score

    def observed(*args, **kwargs):
        scores, ridx, rvalid = original(*args, **kwargs)
        scores.retain_grad()
        seen["scores"] = scores
        return scores, ridx, rvalid

    def partition(grid, batch, mode):
        n = grid[0] * grid[1]
        a_rows, b_rows = [], []
        for bi in range(batch):
            if mode == "alternating":
                tokens = np.arange(n)
                a_tok, b_tok = tokens[(tokens + bi) % 2 == 0], tokens[(tokens + bi) % 2 == 1]
            else:
                perm = rng.permutation(n)
                a_tok, b_tok = np.sort(perm[: n // 2]), np.sort(perm[n // 2:])
            a_rows.append(a_tok + 1)
            b_rows.append(b_tok + 1)
        return torch.from_numpy(np.stack(a_rows)), torch.from_numpy(np.stack(b_rows))

    ref_dtem.sparse_spatial_score = observed
    try:
        for i, (grid, radius, batch, k, channels, mode) in enumerate(
                [((3, 5), 2, 2, 3, 9, "reference_test"), ((8, 8), 3, 2, 16, 16, "alternating"),
                 ((6, 7), 1, 3, 3, 8, "random")]):
            if mode == "reference_test":  # tests/test_dtem_spatial_sparse.py:179-227
                a_idx = torch.tensor([[1, 3, 5, 7, 9, 11, 13], [2, 4, 6, 8, 10, 12, 14]])
                b_idx = torch.tensor([[2, 4, 6, 8, 10, 12, 14, 15], [1, 3, 5, 7, 9, 11, 13, 15]])
            else:
                a_idx, b_idx = partition(grid, batch, mode)
            na, nb = a_idx.shape[1], b_idx.shape[1]
            a = (rng.standard_normal((batch, na, channels), dtype=np.float32) * 0.5).astype(np.float32)
            b = (rng.standard_normal((batch, nb, channels), dtype=np.float32) * 0.5).astype(np.float32)
            block = make_block(grid, radius, "sparse")
            ta = torch.from_numpy(a).requires_grad_(True)
            tb = torch.from_numpy(b).requires_grad_(True)
            assign, _ = block._select(k, ta, tb, a_idx, b_idx)
            g = rng.standard_normal(tuple(assign.shape), dtype=np.float32)
            assign.backward(torch.from_numpy(g))
            scores = seen["scores"]
            cases.update({f"grid{i}": np.array(grid), f"radius{i}": radius, f"k{i}": k,
                          f"a{i}": a, f"b{i}": b, f"a_idx{i}": a_idx.numpy(), f"b_idx{i}": b_idx.numpy(),
                          f"grad_assign{i}": g, f"assign{i}": assign.detach().numpy(),
                          f"scores{i}": scores.detach().numpy(), f"grad_scores{i}": scores.grad.numpy(),
                          f"allowed{i}": block._tome_info["assign_valid_mask"].numpy(),
                          f"grad_a{i}": ta.grad.numpy(), f"grad_b{i}": tb.grad.numpy()})
    finally:
        ref_dtem.sparse_spatial_score = original
    cases["count"] = np.int64(3)
    np.savez_compressed(HERE / "select_backward.npz", **cases)


def merge_train_backward_case():
    """One training-mode soft merge layer of the reference,
    DTEMBlock._merge_train (opentome/timm/dtem.py:1687-2223), differentiated
    by its own autograd: gradients of random upstream gradients on the
    output tokens and masses with respect to x, size and the metric.  The
    deterministic train groupings make the partition reproducible: the
    strided parity split and a seeded permutation (the generic gather /
    scatter path)."""
    rng = np.random.default_rng(20261204)
    cases = {}
    specs = [((8, 8), 3.0, 2, 16, 8, 12, "alternating_per_layer_fast", 1),
             ((6, 7), 2.0, 3, 12, 6, 9, "seeded", 0)]
    for i, (grid, radius, batch, channels, metric_dim, r, grouping, layer) in enumerate(specs):
        t = grid[0] * grid[1] + 1
        x = rng.standard_normal((batch, t, channels), dtype=np.float32)
        metric = rng.standard_normal((batch, t, metric_dim), dtype=np.float32)
        size = (1.0 + 2.0 * rng.random((batch, t, 1))).astype(np.float32)
        block = make_block(grid, radius, "sparse")
        block.train()
        block._tome_info.update({"train_grouping": grouping, "train_grouping_seed": 7, "merge_layer_index": layer})
        tx = torch.from_numpy(x).requires_grad_(True)
        tm = torch.from_numpy(metric).requires_grad_(True)
        ts = torch.from_numpy(size).requires_grad_(True)
        x_out, size_out, _, _, _ = block._merge_train(tx, ts, r, t, {"metric": tm})
        gx = rng.standard_normal(tuple(x_out.shape), dtype=np.float32)
        gs = rng.standard_normal(tuple(size_out.shape), dtype=np.float32)
        torch.autograd.backward([x_out, size_out], [torch.from_numpy(gx), torch.from_numpy(gs)])
        cases.update({f"grid{i}": np.array(grid), f"radius{i}": radius, f"r{i}": r, f"grouping{i}": grouping,
                      f"layer{i}": layer, f"x{i}": x, f"metric{i}": metric, f"size{i}": size,
                      f"x_out{i}": x_out.detach().numpy(), f"size_out{i}": size_out.detach().numpy(),
                      f"center{i}": block._tome_info["token_center"].numpy(),
                      f"grad_x_out{i}": gx, f"grad_size_out{i}": gs, f"grad_x{i}": tx.grad.numpy(),
                      f"grad_metric{i}": tm.grad.numpy(), f"grad_size{i}": ts.grad.numpy()})
    cases["count"] = np.int64(len(specs))
    np.savez_compressed(HERE / "merge_train_backward.npz", **cases)


def merge_train_chain_backward_case():
    """The six training-mode merge layers chained as LocalEncoder.forward
    chains them (model.py:574-590; merge_layer_index per layer, sizes and
    token centres carried), then the carrier block's mass top-k and gather
    (model.py:1157-1183), differentiated by the reference's autograd:
    gradients of random upstream gradients on the final tokens, the final
    masses and the gathered carriers with respect to the input tokens and
    every layer's metric."""
    rng = np.random.default_rng(20261205)
    grid, radius, batch, channels, metric_dim = (8, 8), 3.0, 2, 16, 8
    r_list = canonical_r_list(grid)
    t = grid[0] * grid[1] + 1
    x = rng.standard_normal((batch, t, channels), dtype=np.float32)
    metrics = rng.standard_normal((len(r_list), batch, t, metric_dim), dtype=np.float32)
    block = make_block(grid, radius, "sparse")
    block.train()
    block._tome_info.update({"train_grouping": "alternating_per_layer_fast", "train_grouping_seed": 0})
    tx = torch.from_numpy(x).requires_grad_(True)
    tm = torch.from_numpy(metrics).requires_grad_(True)
    xs, size, n = tx, torch.ones(batch, t, 1), t
    for i, r in enumerate(r_list):
        block._tome_info["merge_layer_index"] = i
        xs, size, n, _, _ = block._merge_train(xs, size, r, n, {"metric": tm[i]})
    k = t - sum(r_list) - 1
    strength = size[..., 0][:, 1:]
    idx = torch.topk(strength.detach(), k, dim=1, largest=True, sorted=False).indices
    order = torch.argsort(torch.gather(block._tome_info["token_center"][:, 1:], 1, idx), dim=1)
    topk = torch.gather(idx, 1, order)
    carriers = torch.gather(xs, 1, (topk + 1).unsqueeze(-1).expand(-1, -1, channels))
    gx = rng.standard_normal(tuple(xs.shape), dtype=np.float32)
    gs = rng.standard_normal(tuple(size.shape), dtype=np.float32)
    gc = rng.standard_normal(tuple(carriers.shape), dtype=np.float32)
    torch.autograd.backward([xs, size, carriers], [torch.from_numpy(gx), torch.from_numpy(gs), torch.from_numpy(gc)])
    np.savez_compressed(HERE / "merge_train_chain_backward.npz", grid=np.array(grid), radius=radius,
                        r_list=np.array(r_list), x=x, metrics=metrics, x_out=xs.detach().numpy(),
                        size_out=size.detach().numpy(), topk_idx=topk.numpy(),
                        center=block._tome_info["token_center"].numpy(), grad_x_out=gx, grad_size_out=gs,
                        grad_carriers=gc, grad_x=tx.grad.numpy(), grad_metrics=tm.grad.numpy())


def neighbor_dot_backward_case():
    """Gradients of the reference's sparse_neighbor_dot (the score of
    sparse_spatial_score too) through its own autograd Function
    (opentome/timm/dtem.py:597-677): grad_a gathers, grad_b scatter-adds
    over the edges in donor-major order.  Random edge lists with repeated
    receivers and invalid slots, as the reference's tests draw them."""
    rng = np.random.default_rng(20261202)
    cases = {}
    for i, (batch, donors, receivers, neighbors, channels) in enumerate(
            [(2, 50, 57, 13, 24), (3, 392, 392, 29, 64)]):
        a = rng.standard_normal((batch, donors, channels), dtype=np.float32)
        b = rng.standard_normal((batch, receivers, channels), dtype=np.float32)
        ridx = rng.integers(0, receivers, (batch, donors, neighbors))
        rvalid = rng.random((batch, donors, neighbors)) > 0.2
        gs = rng.standard_normal((batch, donors, neighbors), dtype=np.float32)
        ta = torch.from_numpy(a).requires_grad_(True)
        tb = torch.from_numpy(b).requires_grad_(True)
        scores = sparse_neighbor_dot(ta, tb, torch.from_numpy(ridx), torch.from_numpy(rvalid))
        scores.backward(torch.from_numpy(gs))
        cases.update({f"a{i}": a, f"b{i}": b, f"receiver_indices{i}": ridx.astype(np.int32),
                      f"receiver_valid{i}": rvalid, f"grad_scores{i}": gs,
                      f"scores{i}": scores.detach().numpy(), f"grad_a{i}": ta.grad.numpy(),
                      f"grad_b{i}": tb.grad.numpy()})
    np.savez_compressed(HERE / "neighbor_dot_backward.npz", **cases)


def attention_case():
    """The reference's own CPU unfold implementations of the windowed
    attention (opentome/timm/bias_local_attn.py:46-240), BNHD layout."""
    rng = np.random.default_rng(20260809)
    cases = {}
    for i, (b, n, h, d, w) in enumerate([(2, 11, 3, 16, 2), (2, 40, 4, 64, 16), (1, 37, 2, 32, 5)]):
        q = (rng.standard_normal((b, n, h, d), dtype=np.float32) * 0.5).astype(np.float32)
        k = (rng.standard_normal((b, n, h, d), dtype=np.float32) * 0.5).astype(np.float32)
        v = rng.standard_normal((b, n, h, d), dtype=np.float32)
        bias = (rng.standard_normal((b, n), dtype=np.float32) * 0.5).astype(np.float32)
        tq, tk, tv, tb = (torch.from_numpy(t) for t in (q, k, v, bias))
        cases[f"q{i}"], cases[f"k{i}"], cases[f"v{i}"], cases[f"bias{i}"] = q, k, v, bias
        cases[f"window{i}"] = w
        cases[f"unbiased{i}"] = naive_unbiased_local_attention(tq, tk, tv, w).numpy()
        cases[f"biased{i}"] = naive_biased_local_attention(tq, tk, tv, tb, w).numpy()
    np.savez_compressed(HERE / "attention.npz", **cases)


def main():
    # `make_golden.py <case> ...` regenerates only the named cases
    only = set(sys.argv[1:])
    if only:
        for name in only:
            globals()[name]()
        return
    attention_case()
    neighbor_dot_backward_case()
    thre_topk_case()
    thre_topk_backward_case()
    select_case()
    select_backward_case()
    merge_train_backward_case()
    merge_train_chain_backward_case()
    transport_case()
    route_case("route_g3x6", 101, 2, (3, 6), 2.0, 7, 5, [3, 3], capture=True)
    route_case("route_g4x4", 102, 3, (4, 4), 1.5, 16, 8, [2, 2, 2], capture=True)
    route_case("route_c1", 0, 2, (28, 28), 3.0, 384, 64, canonical_r_list((28, 28)),
               capture=True, dense_check=True)
    route_case("route_c2_b128", 1, 128, (28, 28), 3.0, 8, 64, canonical_r_list((28, 28)),
               keep_features=False, dense_check=True)
    route_case("route_g48", 5, 2, (48, 48), 3.0, 16, 64, canonical_r_list((48, 48)))


if __name__ == "__main__":
    main()
