"""The numpy oracle against fixtures produced by the reference itself."""
import numpy as np
import pytest

from inputs import canonical_r_list, routing_inputs
from oracle import routing as O

ROUTE_CASES = ["route_g3x6", "route_g4x4", "route_c1", "route_g48", "route_c2_b128"]


def load(golden_dir, name):
    return np.load(golden_dir / f"{name}.npz")


def run_case(g):
    grid = tuple(int(v) for v in g["grid"])
    r_list = [int(v) for v in g["r_list"]]
    x, metrics = routing_inputs(int(g["seed"]), int(g["batch"]), grid, int(g["channels"]),
                                int(g["metric_dim"]), layers=len(r_list))
    geom = O.Geometry(grid, float(g["radius"]))
    return O.route_and_gather(x, metrics, r_list, geom, keep_info=True), r_list


@pytest.mark.parametrize("name", ROUTE_CASES)
def test_oracle_route_matches_reference(golden_dir, name):
    g = load(golden_dir, name)
    out, r_list = run_case(g)
    np.testing.assert_array_equal(out["topk_idx"], g["topk_idx"])
    # the reference's own dense and sparse CPU backends differ by up to 1.4e-5
    np.testing.assert_allclose(out["size"], g["size"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(out["center"], g["center"], rtol=0, atol=2e-3)
    np.testing.assert_allclose(out["topk_size"], g["topk_size"], rtol=3e-5, atol=3e-5)
    if "topk_x" in g:
        np.testing.assert_allclose(out["topk_x"], g["topk_x"], rtol=1e-4, atol=1e-4)
    for i in range(len(r_list)):
        if f"assign_{i}" in g:
            np.testing.assert_allclose(out["layers"][i]["assign"], g[f"assign_{i}"], rtol=0, atol=5e-6)
            np.testing.assert_array_equal(out["layers"][i]["receiver_indices"], g[f"receiver_indices_{i}"])
            np.testing.assert_array_equal(out["layers"][i]["receiver_valid"], g[f"receiver_valid_{i}"])


def test_reference_dense_and_sparse_agree(golden_dir):
    for name in ("route_c1", "route_c2_b128"):
        g = load(golden_dir, name)
        np.testing.assert_array_equal(g["dense_topk_idx"], g["topk_idx"])


def test_oracle_thre_topk(golden_dir):
    g = load(golden_dir, "thre_topk")
    for i in range(4):
        y = O.thre_topk(g[f"x{i}"], int(g[f"k{i}"]))
        np.testing.assert_allclose(y, g[f"y{i}"].reshape(y.shape), rtol=0, atol=2e-6)


def test_oracle_select_and_score(golden_dir):
    g = load(golden_dir, "select_g3x5")
    geom = O.Geometry((3, 5), 2.0)
    scores, ridx, rvalid = O.sparse_spatial_score(g["a"], g["b"], geom.nbr_idx, geom.nbr_valid,
                                                  g["a_idx"] - 1, g["b_idx"] - 1)
    np.testing.assert_allclose(scores, g["scores"], rtol=0, atol=1e-5)
    np.testing.assert_array_equal(ridx, g["receiver_indices"])
    np.testing.assert_array_equal(rvalid, g["receiver_valid"])
    assign, _, _ = O.select(3, scores, rvalid)
    np.testing.assert_allclose(assign, g["assign"], rtol=0, atol=2e-6)


def test_oracle_transport(golden_dir):
    g = load(golden_dir, "transport")
    out = O.sparse_weighted_transport(g["assignment"], g["values"], g["receiver_indices"], g["receiver_valid"],
                                      int(g["receivers"]))
    np.testing.assert_allclose(out, g["out"], rtol=1e-6, atol=1e-6)


def test_oracle_budget_fails_closed():
    geom = O.Geometry((1, 4), 0.5)
    a = np.random.default_rng(0).standard_normal((1, 2, 4)).astype(np.float32)
    scores, ridx, rvalid = O.sparse_spatial_score(a, a, geom.nbr_idx, geom.nbr_valid,
                                                  np.array([[0, 2]]), np.array([[1, 3]]))
    assert not rvalid.any()
    with pytest.raises(RuntimeError):
        O.select(1, scores, rvalid)


def test_parse_r_schedule():
    assert O.parse_r(6, 65, 392) == [65, 65, 65, 65, 65, 67]
    assert canonical_r_list((28, 28)) == [65, 65, 65, 65, 65, 67]
    assert canonical_r_list((48, 48)) == [192] * 6
    assert O.parse_r(3, [1, 2]) == [1, 2, 0]


def test_oracle_attention_matches_reference_naive(golden_dir):
    """oracle/attention.py against the reference's unfold implementations
    (naive_unbiased_local_attention / naive_biased_local_attention) on all
    three fixture cases; those take a pre-scaled q, so the scale is 1."""
    from oracle.attention import local_attention
    g = np.load(golden_dir / "attention.npz")
    for i in range(3):
        q, k, v, bias = (g[f"{n}{i}"] for n in ("q", "k", "v", "bias"))
        w = int(g[f"window{i}"])
        np.testing.assert_allclose(local_attention(q, k, v, w, scale=1.0), g[f"unbiased{i}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(local_attention(q, k, v, w, bias=bias, scale=1.0), g[f"biased{i}"],
                                   rtol=1e-5, atol=1e-5)


def test_timed_port_routing_matches_the_oracle():
    """The batched torch routing of the timed CPU baseline (model_cpu.route_torch)
    gives the oracle's carriers, masses and features."""
    import torch
    from oracle import model_cpu
    grid = (28, 28)
    r_list = canonical_r_list(grid)
    x, metrics = routing_inputs(3, 2, grid, 32, 64)
    geom = O.Geometry(grid, 3.0)
    ref = O.route_and_gather(x, metrics, r_list, geom)
    tx, ts, ti = model_cpu.route_torch(torch.from_numpy(x), [torch.from_numpy(m.astype(np.float32)) for m in metrics],
                                       r_list, geom)
    np.testing.assert_array_equal(ti.numpy(), ref["topk_idx"])
    np.testing.assert_allclose(ts.numpy(), ref["topk_size"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(tx.numpy(), ref["topk_x"], rtol=1e-4, atol=1e-4)


def test_oracle_neighbor_dot_backward(golden_dir):
    """The restated gradients against the reference's own autograd run."""
    g = load(golden_dir, "neighbor_dot_backward")
    for i in range(2):
        ga, gb = O.sparse_neighbor_dot_backward(g[f"a{i}"], g[f"b{i}"], g[f"receiver_indices{i}"],
                                                g[f"receiver_valid{i}"], g[f"grad_scores{i}"])
        np.testing.assert_allclose(ga, g[f"grad_a{i}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(gb, g[f"grad_b{i}"], rtol=1e-5, atol=1e-5)
        s = O.sparse_neighbor_dot(g[f"a{i}"], g[f"b{i}"], g[f"receiver_indices{i}"], g[f"receiver_valid{i}"])
        np.testing.assert_allclose(s, g[f"scores{i}"], rtol=1e-5, atol=1e-5)


def test_oracle_thre_topk_backward(golden_dir):
    """The closed-form ThreTopK gradient against the reference's autograd."""
    g = load(golden_dir, "thre_topk_backward")
    for i in range(int(g["count"])):
        dx = O.thre_topk_backward(g[f"x{i}"], int(g[f"k{i}"]), g[f"g{i}"])
        ref = g[f"dx{i}"]
        assert np.abs(dx - ref).max() <= 2e-5 * np.abs(ref).max()


def test_oracle_select_backward(golden_dir):
    """The select block's score gradient against the reference's autograd
    through DTEMBlock._select (observed at its sparse_spatial_score call)."""
    g = load(golden_dir, "select_backward")
    for i in range(int(g["count"])):
        ds = O.select_backward(int(g[f"k{i}"]), g[f"scores{i}"], g[f"allowed{i}"], g[f"grad_assign{i}"])
        ref = g[f"grad_scores{i}"]
        assert np.abs(ds - ref).max() <= 2e-5 * np.abs(ref).max(), i
