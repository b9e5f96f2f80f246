"""Host-side checks of libmergenet_b200.so that need no GPU: it loads, it
exports every entry point the header declares, and its host geometry matches
the oracle (and through it the reference's own tests)."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import routing as O

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_every_header_symbol():
    from mergenet_b200 import _lib
    lib = _lib.lib()
    header = (ROOT / "include" / "mergenet_b200.h").read_text()
    declared = set(re.findall(r"^(?:int|size_t)\s+(mn_\w+)\s*\(", header, flags=re.M))
    assert declared, "no declarations parsed"
    assert declared == set(_lib.EXPORTED), declared ^ set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.mn_version() == 1


@pytest.mark.parametrize("grid,radius", [((28, 28), 3.0), ((48, 48), 3.0), ((3, 5), 1.5), ((2, 3), 1.0),
                                         ((3, 6), 2.0), ((4, 4), 1.5), ((1, 4), 0.5), ((3, 5), 4.47213595499958)])
def test_neighbor_table_matches_oracle(grid, radius):
    import mergenet_b200 as mn
    idx, val = mn.build_patch_spatial_neighbors(grid, radius)
    geom = O.Geometry(grid, radius)
    np.testing.assert_array_equal(idx.numpy(), geom.nbr_idx)
    np.testing.assert_array_equal(val.numpy(), geom.nbr_valid)
    adj = mn.build_patch_spatial_adjacency(grid, radius)
    np.testing.assert_array_equal(adj.numpy(), geom.adjacency)


def test_reference_geometry_facts():
    """tests/test_dtem_spatial_sparse.py:50-65 and test_dtem_spatial_mask.py:32-63."""
    import mergenet_b200 as mn
    idx, val = mn.build_patch_spatial_neighbors((3, 5), 1.5)
    assert idx.shape == val.shape == (15, 9)
    assert int(val[0].sum()) == 4
    adj = mn.build_patch_spatial_adjacency((3, 5), 1.5)
    assert not bool(adj[4, 5]) and bool(adj[4, 9])
    adj = mn.build_patch_spatial_adjacency((2, 3), 1)
    assert not bool(adj[2, 3]) and bool(adj[0, 3]) and bool(torch.diagonal(adj).all())
    assert bool(mn.build_patch_spatial_adjacency((3, 5), float(np.hypot(2, 4))).all())
    idx, val = mn.build_patch_spatial_neighbors((28, 28), 3.0)
    assert idx.shape == (784, 29) and int(val.sum()) == 20756
    counts = val.sum(1)
    assert int(counts.min()) == 11 and int(counts.max()) == 29
    _, val = mn.build_patch_spatial_neighbors((48, 48), 3.0)
    assert int(val.sum()) == 63396


@pytest.mark.parametrize("grid", [0, -1, (0, 3), (2, 0), (2.0, 3), (2,), (2, 3, 4)])
def test_invalid_grid_fails_closed(grid):
    import mergenet_b200 as mn
    with pytest.raises(ValueError):
        mn.build_patch_spatial_neighbors(grid, 1.0)


@pytest.mark.parametrize("radius", [-1, float("nan"), 0.0, True])
def test_invalid_radius_fails_closed(radius):
    import mergenet_b200 as mn
    with pytest.raises(ValueError):
        mn.build_patch_spatial_neighbors((2, 3), radius)


def _route_tables(grid, radius):
    from mergenet_b200 import _lib
    lib = _lib.lib()
    dims = _lib.RouteDims()
    assert lib.mn_route_dims_query(grid[0], grid[1], radius, ctypes.byref(dims)) == 0
    table = np.zeros(dims.table_ints, np.int32)
    assert lib.mn_route_tables_fill(grid[0], grid[1], radius, ctypes.byref(dims),
                                    table.ctypes.data_as(ctypes.c_void_p)) == 0
    return dims, table


@pytest.mark.parametrize("grid,radius", [((28, 28), 3.0), ((48, 48), 3.0), ((3, 6), 2.0), ((4, 4), 1.5)])
def test_route_tables_match_sparse_mapping(grid, radius):
    """Compact donor slots and receiver in-lists agree with the reference's
    sorted-receiver mapping (dtem.py:219-234) for both layer parities."""
    dims, table = _route_tables(grid, radius)
    geom = O.Geometry(grid, radius)
    half, kc, kin = dims.half, dims.kc, dims.kin
    p = grid[0] * grid[1]
    per = half * kc * 2 + half * kin * 2
    w = grid[1]
    # stencil order: odd dx ascending, then dy ascending within each |dx| limit
    offsets = [(dy, dx) for dx in (-3, -1, 1, 3)
               for dy in range(-(dims.stencil_dy3 if abs(dx) == 3 else dims.stencil_dy1),
                               (dims.stencil_dy3 if abs(dx) == 3 else dims.stencil_dy1) + 1)]
    for q in (0, 1):
        dp = 0 if q else 1
        t = table[q * per:(q + 1) * per]
        slot_k = t[:half * kc].reshape(half, kc)
        slot_rx = t[half * kc:2 * half * kc].reshape(half, kc)
        rx_in = t[2 * half * kc:2 * half * kc + half * kin].reshape(half, kin)
        rx_off = t[2 * half * kc + half * kin:].reshape(half, kin)
        for s_ in range(half):
            for j in np.nonzero(rx_in[s_] >= 0)[0]:
                d = rx_in[s_, j] // kc
                pd, ps = 2 * d + dp, 2 * s_ + (1 - dp)
                assert offsets[rx_off[s_, j]] == (pd // w - ps // w, pd % w - ps % w)
        donors = np.arange(dp, p, 2)[None]
        recv = np.arange(1 - dp, p, 2)[None]
        ridx, rvalid = O.map_sorted_receivers(geom.nbr_idx, geom.nbr_valid, donors, recv)
        edges = []
        for d in range(half):
            ks = np.nonzero(rvalid[0, d])[0]
            got = slot_k[d][slot_k[d] >= 0]
            np.testing.assert_array_equal(got, ks)
            np.testing.assert_array_equal(slot_rx[d][: len(ks)], ridx[0, d, ks])
            edges += [(int(ridx[0, d, k]), d * kc + c) for c, k in enumerate(ks)]
        for s in range(half):
            want = [e for r, e in edges if r == s]  # donor-major order = sequential scatter order
            got = rx_in[s][rx_in[s] >= 0].tolist()
            assert got == want
        assert dims.valid_rows[q] == int(rvalid[0].any(-1).sum())
    if grid == (28, 28):
        assert (dims.kc, dims.kin, dims.k_static) == (12, 12, 29)
        assert (dims.stencil_dy1, dims.stencil_dy3) == (2, 0)


def test_cpu_tensors_are_rejected():
    """No CPU fallback: the product path refuses host tensors loudly."""
    import mergenet_b200 as mn
    with pytest.raises(RuntimeError):
        mn.ThreTopK(torch.rand(2, 5), 2)
    with pytest.raises(RuntimeError):
        mn.unbiased_local_attention(torch.rand(1, 5, 2, 64), torch.rand(1, 5, 2, 64), torch.rand(1, 5, 2, 64), 1)


def test_training_functions_refuse_host_tensors():
    """The gradient entry points and the carrier block's training terms have
    no CPU path either: host tensors, with or without autograd, raise before
    any kernel is launched."""
    import mergenet_b200 as mn
    x = torch.rand(2, 8)
    with pytest.raises(RuntimeError):
        mn.thre_topk_backward(x, 3, torch.rand(2, 8))
    with pytest.raises(RuntimeError):
        mn.ThreTopK(x.clone().requires_grad_(True), 3)
    scores, allowed = torch.rand(1, 4, 3), torch.ones(1, 4, 3, dtype=torch.bool)
    with pytest.raises(RuntimeError):
        mn.dtem_select_backward(2, scores, allowed, torch.rand(1, 4, 3))
    with pytest.raises(RuntimeError):
        mn.dtem_select(2, scores.clone().requires_grad_(True), allowed)
    with pytest.raises(RuntimeError):
        mn.soft_topk_aux_repr(torch.rand(2, 8, 4), x)
    with pytest.raises(RuntimeError):
        mn.carrier_ste(torch.rand(2, 3, 4), x, torch.zeros(2, 3, dtype=torch.long))
    with pytest.raises(RuntimeError):
        mn.carrier_ste(torch.rand(2, 3, 4), x.clone().requires_grad_(True), torch.zeros(2, 3, dtype=torch.long))


def test_attention_argument_checks_precede_any_launch():
    """A per-key bias that is not (B, N) and a packed width that is not
    3 x heads x head_dim are refused before the device is touched, so the
    kernels never index past the bias; well-formed host tensors still meet
    the no-CPU-path error."""
    import mergenet_b200 as mn
    qkv = torch.rand(2, 7, 3 * 2 * 64)
    with pytest.raises(ValueError, match="bias must be"):
        mn.local_attention_packed(qkv, 2, 1, bias=torch.rand(2, 6))
    with pytest.raises(ValueError, match="bias must be"):
        mn.local_attention_packed(qkv, 2, 1, bias=torch.rand(7, 2))
    with pytest.raises(ValueError, match="packed qkv width"):
        mn.local_attention_packed(torch.rand(2, 7, 40), 2, 1)
    with pytest.raises(RuntimeError):
        mn.local_attention_packed(qkv, 2, 1, bias=torch.rand(2, 7))


def test_attention_shapes_outside_the_kernels_are_refused():
    """One backend: head_dim other than 64 is a ValueError before any device
    work, and so is the reference's generic-path case logical_dim < head_dim
    with head_dim % 8 != 0 (it would return head_dim columns there)."""
    import mergenet_b200 as mn
    t = torch.rand(1, 9, 2, 16)
    with pytest.raises(ValueError, match="head_dim 16"):
        mn.unbiased_local_attention(t, t, t, 2)
    t65 = torch.rand(1, 9, 2, 65)
    with pytest.raises(ValueError, match="head_dim % 8"):
        mn.biased_local_attention(t65, t65, t65, torch.rand(1, 9), 2, logical_dim=64, input_layout="BNHD")
    with pytest.raises(ValueError, match="head_dim 32"):
        mn.cross_attention(torch.rand(1, 3, 2, 32), torch.rand(1, 5, 2, 32), torch.rand(1, 5, 2, 32))


def test_merge_block_refuses_paths_it_does_not_implement():
    """DTEMMergeBlock covers the sparse spatial soft-k-max path in eval and
    training mode; the other paths, and train groupings the reference does
    not have, are refused before any device work."""
    import mergenet_b200 as mn
    block = mn.DTEMMergeBlock({"window_size": 0, "dtem_spatial_radius": 3.0, "dtem_spatial_backend": "sparse",
                               "tau2": 30.0, "train_grouping": "random"})
    x = torch.zeros(1, 5, 8)
    size = torch.ones(1, 5, 1)
    with pytest.raises(ValueError, match="grouping"):
        block.train()._merge_train(x, size, 1, 5, {"metric": torch.ones(1, 5, 4)})
    block.eval()
    block._tome_info["dtem_spatial_backend"] = "dense"
    with pytest.raises(NotImplementedError, match="sparse backend"):
        block._merge_train(x, size, 1, 5, {"metric": torch.ones(1, 5, 4)})
    block._tome_info.update(dtem_spatial_backend="sparse", source_trace_mode="matrix")
    with pytest.raises(NotImplementedError, match="source"):
        block._merge_train(x, size, 1, 5, {"metric": torch.ones(1, 5, 4)})


def test_eval_group_indices_follow_the_layer_parity():
    """build_dtem_eval_group_indices (dtem.py:1125-1188): even layers donate
    the odd positions, odd layers the even ones; 'seeded' is batch-shared."""
    import mergenet_b200 as mn
    a0, b0 = mn.build_eval_group_indices(6, 2, "cpu", "alternating_per_layer", layer_index=0)
    a1, b1 = mn.build_eval_group_indices(6, 2, "cpu", "alternating_per_layer_fast", layer_index=1)
    assert a0[0].tolist() == [1, 3, 5] and b0[0].tolist() == [0, 2, 4]
    assert a1[0].tolist() == [0, 2, 4] and b1[0].tolist() == [1, 3, 5]
    s0, _ = mn.build_eval_group_indices(10, 3, "cpu", "seeded", seed=4, layer_index=2)
    assert torch.equal(s0[0], s0[2])
    with pytest.raises(ValueError):
        mn.build_eval_group_indices(6, 2, "cpu", "random")


def test_state_dict_matches_the_reference_model(golden_dir):
    """The reference's own mergenet_small_cls (built by make_model_golden.py)
    has exactly our parameter names and shapes, so its checkpoints load with
    strict=True; the geometry buffers are not persistent, as in the
    reference (model.py:350-364)."""
    import numpy as np
    from inputs import model_weights
    from mergenet_b200.model import mergenet_small_cls
    g = np.load(golden_dir / "model_small_cls.npz")
    ref = dict(zip(g["param_names"].tolist(), g["param_shapes"].tolist()))
    model = mergenet_small_cls()
    ours = {k: ",".join(map(str, tuple(v.shape))) for k, v in model.state_dict().items()}
    assert ours == ref
    weights = model_weights({k: tuple(int(x) for x in v.split(",")) for k, v in ref.items()}, seed=0)
    model.load_state_dict({k: torch.from_numpy(v) for k, v in weights.items()}, strict=True)


def test_factory_accepts_the_reference_kwargs_and_refuses_other_paths():
    from mergenet_b200.model import MERGENET_SMALL_CANONICAL_KWARGS, mergenet_small_cls
    m = mergenet_small_cls(num_classes=10, **MERGENET_SMALL_CANONICAL_KWARGS)
    assert m.grid == (28, 28) and m.r_list == [65, 65, 65, 65, 65, 67] and m.local_window == 16
    m48 = mergenet_small_cls(img_size=384)
    assert m48.grid == (48, 48) and m48.r_list == [192] * 6
    with pytest.raises(NotImplementedError):
        mergenet_small_cls(total_merge_latent=4)
    with pytest.raises(NotImplementedError):
        mergenet_small_cls(dtem_window_size=8)
    with pytest.raises(TypeError):
        mergenet_small_cls(not_an_argument=1)


def test_merge_block_groupings_follow_the_mode():
    """DTEMMergeBlock picks its donor / receiver split as dtem.py:1755-1812
    does: eval mode from eval_grouping / eval_grouping_seed, training mode
    from train_grouping / train_grouping_seed (the strided split only for
    alternating_per_layer_fast with an even token count), and the default
    training grouping draws a fresh permutation per image."""
    import mergenet_b200 as mn
    block = mn.DTEMMergeBlock({"eval_grouping": "seeded", "eval_grouping_seed": 3, "train_grouping": "seeded",
                               "train_grouping_seed": 9, "merge_layer_index": 2})
    a_e, b_e, strided = block.eval()._groups(10, 2, "cpu")
    want_a, want_b = mn.build_eval_group_indices(10, 2, "cpu", "seeded", seed=3, layer_index=2)
    assert not strided and torch.equal(a_e, want_a) and torch.equal(b_e, want_b)
    a_t, b_t, strided = block.train()._groups(10, 2, "cpu")
    want_a, want_b = mn.build_eval_group_indices(10, 2, "cpu", "seeded", seed=9, layer_index=2)
    assert not strided and torch.equal(a_t, want_a) and torch.equal(b_t, want_b)
    block._tome_info["train_grouping"] = "alternating_per_layer_fast"
    assert block._groups(10, 2, "cpu")[2] and not block._groups(9, 2, "cpu")[2]
    block._tome_info["train_grouping"] = "random_per_sample"
    torch.manual_seed(0)
    a_r, b_r, strided = block._groups(10, 3, "cpu")
    assert not strided and a_r.shape == (3, 5) and b_r.shape == (3, 5)
    for i in range(3):  # each image's halves partition the tokens
        assert sorted(torch.cat([a_r[i], b_r[i]]).tolist()) == list(range(10))
    assert any(not torch.equal(a_r[0], a_r[i]) for i in (1, 2))
