"""DTEM spatial routing on the B200 kernels: drop-ins for the reference's
routing functions plus the fused six-layer route-and-gather.

Function names, argument order and meaning follow opentome/timm/dtem.py and
opentome/utils/thetopk.py; every function takes and returns torch tensors on a
CUDA device and launches on the current stream.  There is no CPU path.
"""
from __future__ import annotations

import ctypes
import math
import operator
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L

EPS32 = torch.finfo(torch.float32).eps


# --------------------------------------------------------------------------
# Geometry (dtem.py:50-143)
# --------------------------------------------------------------------------
def _check_grid(grid_size, radius):
    if not isinstance(grid_size, (tuple, list, torch.Size)) or len(grid_size) != 2:
        raise ValueError(f"grid_size must be a (height, width) pair, got {grid_size!r}")
    if any(isinstance(v, bool) for v in grid_size):
        raise ValueError(f"grid_size values must be integers, got {grid_size!r}")
    try:
        h, w = operator.index(grid_size[0]), operator.index(grid_size[1])
    except TypeError as exc:
        raise ValueError(f"grid_size values must be integers, got {grid_size!r}") from exc
    if h <= 0 or w <= 0:
        raise ValueError(f"grid_size values must be positive, got {(h, w)!r}")
    if isinstance(radius, bool):
        raise ValueError("radius must be a positive finite number, not bool")
    radius = float(radius)
    if not math.isfinite(radius) or radius <= 0:
        raise ValueError(f"radius must be a positive finite number, got {radius!r}")
    return h, w, radius


def build_patch_spatial_neighbors(grid_size, radius, metric="euclidean", device=None):
    """Padded [P, K] neighbour table (indices int64, valid bool), ascending
    patch order, built by the library's host geometry (dtem.py:130-143)."""
    if metric != "euclidean":
        raise ValueError(f"Unsupported DTEM spatial metric {metric!r}; expected one of ('euclidean',)")
    h, w, radius = _check_grid(grid_size, radius)
    lib = L.lib()
    k = ctypes.c_int()
    L.check(lib.mn_neighbor_table_width(h, w, radius, ctypes.byref(k)), "mn_neighbor_table_width")
    idx = np.zeros((h * w, k.value), np.int64)
    val = np.zeros((h * w, k.value), np.uint8)
    L.check(lib.mn_neighbor_table_fill(h, w, radius, k.value, idx.ctypes.data_as(ctypes.c_void_p),
                                       val.ctypes.data_as(ctypes.c_void_p)), "mn_neighbor_table_fill")
    return (torch.from_numpy(idx).to(device), torch.from_numpy(val.astype(bool)).to(device))


def build_patch_spatial_adjacency(grid_size, radius, metric="euclidean", device=None):
    """Dense [P, P] bool adjacency (dtem.py:50-92), from the neighbour table."""
    idx, val = build_patch_spatial_neighbors(grid_size, radius, metric, device="cpu")
    p = idx.shape[0]
    adj = torch.zeros(p, p, dtype=torch.bool)
    rows = torch.arange(p)[:, None].expand_as(idx)
    adj[rows[val], idx[val]] = True
    return adj.to(device)


# --------------------------------------------------------------------------
# Function-level drop-ins
# --------------------------------------------------------------------------
def _contig(*ts):
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError("mergenet_b200 kernels take contiguous tensors")


def _as_u8(t):
    return t.view(torch.uint8) if t.dtype == torch.bool else t


def _neighbor_dot_grads(ctx, a, b, ridx, rval, grad_scores):
    """Gradients of scores[d, k] = a[d] . b[r(d, k)] (dtem.py:667-676):
    grad_b is the transport of grad_scores * a into the receivers (the same
    edge-ordered, atomics-free sum as sparse_weighted_transport, which is the
    reference's sequential scatter-add), grad_a the transport adjoint's
    per-donor gather of grad_scores * b.  Invalid slots contribute nothing."""
    g = grad_scores.to(a.dtype).contiguous()
    grad_a = grad_b = None
    if ctx.needs_input_grad[0]:
        grad_a = sparse_transport_adjoint(g, a, ridx, rval, b)[1]
    if ctx.needs_input_grad[1]:
        grad_b = sparse_weighted_transport(g, a, ridx, rval, b.shape[1])
    return grad_a, grad_b


class _SparseNeighborDotFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, receiver_indices, receiver_valid):
        out = _sparse_neighbor_dot(a, b, receiver_indices, receiver_valid)
        ctx.save_for_backward(a.contiguous(), b.contiguous(), receiver_indices.long().contiguous(),
                              receiver_valid.bool().contiguous())
        return out

    @staticmethod
    def backward(ctx, grad_scores):
        a, b, ridx, rval = ctx.saved_tensors
        grad_a, grad_b = _neighbor_dot_grads(ctx, a, b, ridx, rval, grad_scores)
        return grad_a, grad_b, None, None


class _SparseSpatialScoreFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, neighbor_patch_indices, neighbor_patch_valid, donor_patch_indices,
                receiver_patch_indices):
        scores, ridx, rval = _sparse_spatial_score(a, b, neighbor_patch_indices, neighbor_patch_valid,
                                                   donor_patch_indices, receiver_patch_indices)
        ctx.save_for_backward(a.contiguous(), b.contiguous(), ridx, rval)
        ctx.mark_non_differentiable(ridx, rval)
        return scores, ridx, rval

    @staticmethod
    def backward(ctx, grad_scores, _grad_indices, _grad_valid):
        a, b, ridx, rval = ctx.saved_tensors
        grad_a, grad_b = _neighbor_dot_grads(ctx, a, b, ridx, rval, grad_scores)
        return grad_a, grad_b, None, None, None, None


def _wants_grad(*tensors):
    return torch.is_grad_enabled() and any(t.requires_grad for t in tensors)


def sparse_spatial_score(a, b, neighbor_patch_indices, neighbor_patch_valid, donor_patch_indices,
                         receiver_patch_indices):
    """(scores [B,Na,K], receiver_indices int64 [B,Na,K], receiver_valid bool
    [B,Na,K]) exactly as dtem.py:813-848; receivers must be sorted per row.
    Differentiable in a and b (_SparseSpatialScore.backward, dtem.py:768-810)."""
    if _wants_grad(a, b):
        return _SparseSpatialScoreFn.apply(a, b, neighbor_patch_indices, neighbor_patch_valid, donor_patch_indices,
                                           receiver_patch_indices)
    return _sparse_spatial_score(a, b, neighbor_patch_indices, neighbor_patch_valid, donor_patch_indices,
                                 receiver_patch_indices)


def _sparse_spatial_score(a, b, neighbor_patch_indices, neighbor_patch_valid, donor_patch_indices,
                          receiver_patch_indices):
    dev = L.require_cuda(a, b, neighbor_patch_indices, neighbor_patch_valid, donor_patch_indices,
                         receiver_patch_indices)
    if a.ndim != 3 or b.ndim != 3 or a.shape[0] != b.shape[0] or a.shape[-1] != b.shape[-1]:
        raise ValueError("a and b must have shape [B, N, C] with matching batch/channels")
    if a.dtype != b.dtype:
        raise ValueError("a and b must share a dtype")
    nbr = neighbor_patch_indices.long().contiguous()
    nval = neighbor_patch_valid.bool().contiguous()
    dpat = donor_patch_indices.long().contiguous()
    rpat = receiver_patch_indices.long().contiguous()
    a, b = a.contiguous(), b.contiguous()
    bsz, na, c = a.shape
    nb = b.shape[1]
    p, k = nbr.shape
    scores = torch.empty(bsz, na, k, device=dev, dtype=a.dtype)
    ridx = torch.empty(bsz, na, k, device=dev, dtype=torch.long)
    rval = torch.empty(bsz, na, k, device=dev, dtype=torch.bool)
    L.check(L.lib().mn_sparse_spatial_score(bsz, na, nb, p, k, c, L.dtype_code(a.dtype), L.ptr(a), L.ptr(b),
                                            L.ptr(nbr), L.ptr(_as_u8(nval)), L.ptr(dpat), L.ptr(rpat),
                                            L.ptr(scores), L.ptr(ridx), L.ptr(_as_u8(rval)), L.stream_of(a)),
            "sparse_spatial_score")
    return scores, ridx, rval


def sparse_neighbor_dot(a, b, receiver_indices, receiver_valid):
    """Indexed donor/receiver dot products (dtem.py:680-687), differentiable in
    a and b (_SparseNeighborDot.backward, dtem.py:633-677)."""
    if _wants_grad(a, b):
        return _SparseNeighborDotFn.apply(a, b, receiver_indices, receiver_valid)
    return _sparse_neighbor_dot(a, b, receiver_indices, receiver_valid)


def _sparse_neighbor_dot(a, b, receiver_indices, receiver_valid):
    dev = L.require_cuda(a, b, receiver_indices, receiver_valid)
    if a.dtype != b.dtype:
        raise ValueError("a and b must share a dtype")
    a, b = a.contiguous(), b.contiguous()
    ridx = receiver_indices.long().contiguous()
    rval = receiver_valid.bool().contiguous()
    bsz, na, c = a.shape
    k = ridx.shape[-1]
    out = torch.empty(bsz, na, k, device=dev, dtype=a.dtype)
    L.check(L.lib().mn_sparse_neighbor_dot(bsz, na, b.shape[1], k, c, L.dtype_code(a.dtype), L.ptr(a), L.ptr(b),
                                           L.ptr(ridx), L.ptr(_as_u8(rval)), L.ptr(out), L.stream_of(a)),
            "sparse_neighbor_dot")
    return out


def sparse_weighted_transport(assignment, values, receiver_indices, receiver_valid, num_receivers):
    """out[b, s] = sum of assignment * values over edges into receiver s
    (dtem.py:1035-1067), accumulated in edge order without atomics.
    Differentiable in assignment and values like the reference's
    _SparseTransport (dtem.py:934-974): the backward is
    sparse_transport_adjoint."""
    if _wants_grad(assignment, values):
        return _SparseTransportFn.apply(assignment, values, receiver_indices, receiver_valid, int(num_receivers))
    return _sparse_weighted_transport(assignment, values, receiver_indices, receiver_valid, num_receivers)


class _SparseTransportFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, assignment, values, receiver_indices, receiver_valid, num_receivers):
        out = _sparse_weighted_transport(assignment, values, receiver_indices, receiver_valid, num_receivers)
        a = assignment.contiguous()
        ctx.save_for_backward(a, values.to(a.dtype).contiguous(), receiver_indices.long().contiguous(),
                              receiver_valid.bool().contiguous())
        ctx.values_dtype = values.dtype
        return out

    @staticmethod
    def backward(ctx, grad_output):
        a, v, ridx, rval = ctx.saved_tensors
        gw, gv = sparse_transport_adjoint(a, v, ridx, rval, grad_output.to(v.dtype))
        grad_a = gw if ctx.needs_input_grad[0] else None
        grad_v = gv.to(ctx.values_dtype) if ctx.needs_input_grad[1] else None
        return grad_a, grad_v, None, None, None


def _sparse_weighted_transport(assignment, values, receiver_indices, receiver_valid, num_receivers):
    dev = L.require_cuda(assignment, values, receiver_indices, receiver_valid)
    num_receivers = int(num_receivers)
    if assignment.dtype != values.dtype:
        values = values.to(assignment.dtype)
    assignment, values = assignment.contiguous(), values.contiguous()
    ridx = receiver_indices.long().contiguous()
    rval = receiver_valid.bool().contiguous()
    bsz, na, k = assignment.shape
    c = values.shape[-1]
    out = torch.empty(bsz, num_receivers, c, device=dev, dtype=values.dtype)
    L.check(L.lib().mn_sparse_weighted_transport(bsz, na, num_receivers, k, c, L.dtype_code(values.dtype),
                                                 L.ptr(assignment), L.ptr(values), L.ptr(ridx),
                                                 L.ptr(_as_u8(rval)), L.ptr(out), None, L.stream_of(values)),
            "sparse_weighted_transport")
    return out


def sparse_weighted_transport_pair(assignment, weighted_features, donor_mass, receiver_indices, receiver_valid,
                                   num_receivers):
    """Features and mass with one shared assignment (dtem.py:1006-1032)."""
    features = sparse_weighted_transport(assignment, weighted_features, receiver_indices, receiver_valid,
                                         num_receivers)
    mass = sparse_weighted_transport(assignment, donor_mass.unsqueeze(-1), receiver_indices, receiver_valid,
                                     num_receivers).squeeze(-1)
    return features, mass


def sparse_transport_adjoint(assignment, values, receiver_indices, receiver_valid, grad_output):
    """(grad_assignment, grad_values) of the transport (dtem.py:962-973)."""
    dev = L.require_cuda(assignment, values, receiver_indices, receiver_valid, grad_output)
    assignment, values, grad_output = assignment.contiguous(), values.contiguous(), grad_output.contiguous()
    ridx = receiver_indices.long().contiguous()
    rval = receiver_valid.bool().contiguous()
    bsz, na, k = assignment.shape
    c = values.shape[-1]
    gw = torch.empty_like(assignment)
    gv = torch.empty_like(values)
    L.check(L.lib().mn_sparse_transport_adjoint(bsz, na, grad_output.shape[1], k, c, L.dtype_code(values.dtype),
                                                L.ptr(assignment), L.ptr(values), L.ptr(ridx), L.ptr(_as_u8(rval)),
                                                L.ptr(grad_output), L.ptr(gw), L.ptr(gv), L.stream_of(values)),
            "sparse_transport_adjoint")
    del dev
    return gw, gv


def _status(dev):
    return torch.zeros(1, dtype=torch.int32, device=dev)


def _raise_status(status, what):
    s = int(status.item())
    if s & L.MN_STATUS_INFEASIBLE_BUDGET:
        raise RuntimeError(f"{what}: DTEM spatial radius leaves fewer eligible donor rows than the required "
                           "merge budget")
    if s & L.MN_STATUS_TOO_MANY_EDGES:
        raise ValueError(f"{what}: receiver index out of range")
    if s & L.MN_STATUS_DEGENERATE_RANGE:
        raise RuntimeError(f"{what}: ThreTopK energy range is empty or not finite (global max == min); "
                           "the soft top-k threshold is undefined")
    if s:
        raise RuntimeError(f"{what}: device status {s:#x}")


def _default_check(check):
    """check=None: read the status word now unless a CUDA graph is being
    captured (then the caller reads it after the replay)."""
    if check is None:
        return not torch.cuda.is_current_stream_capturing()
    return bool(check)


def ThreTopK(x, k, temperature=30.0):  # noqa: N802 - reference name
    """Threshold soft top-k (opentome/utils/thetopk.py:4-43): one global
    max - min range over the whole input, per-row threshold.  Differentiable
    in x (thre_topk_backward)."""
    if _wants_grad(x):
        return _ThreTopKFn.apply(x, int(k), float(temperature))
    return _thre_topk(x, k, temperature)


class _ThreTopKFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, k, temperature):
        ctx.save_for_backward(x)
        ctx.k, ctx.temperature = k, temperature
        return _thre_topk(x, k, temperature)

    @staticmethod
    def backward(ctx, grad_y):
        (x,) = ctx.saved_tensors
        return thre_topk_backward(x, ctx.k, grad_y, ctx.temperature), None, None


def thre_topk_backward(x, k, grad_y, temperature=30.0):
    """d ThreTopK(x) / dx applied to grad_y, as the reference's autograd
    differentiates thetopk.py:4-43: through the threshold lambda of the
    row's bracket (its lse1, lse2 and |term|), the two-sided map, the scaled
    input x / R * T and the global range R = max - min, whose gradient is
    split evenly over tied maxima and minima.  Returns grad_x shaped and
    typed like x."""
    dev = L.require_cuda(x, grad_y)
    x32 = x.float().contiguous()
    if x32.dim() == 1:
        x32 = x32.unsqueeze(0)
    rows, n = x32.shape
    g32 = grad_y.float().contiguous().reshape(rows, n)
    gx = torch.empty_like(x32)
    wsb = L.lib().mn_thre_topk_backward_workspace_bytes(rows, n)
    ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device=dev)
    L.check(L.lib().mn_thre_topk_backward(rows, n, L.ptr(x32), int(k), float(temperature), L.ptr(g32), L.ptr(gx),
                                          L.ptr(ws), wsb, None, L.stream_of(x32)), "ThreTopK backward")
    return gx.reshape(x.shape).to(x.dtype)


def _thre_topk(x, k, temperature):
    dev = L.require_cuda(x)
    if x.dim() == 1:
        x = x.unsqueeze(0)
    x32 = x.float().contiguous()
    rows, n = x32.shape
    y = torch.empty_like(x32)
    wsb = L.lib().mn_thre_topk_workspace_bytes(rows, n)
    ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device=dev)
    L.check(L.lib().mn_thre_topk(rows, n, L.ptr(x32), int(k), float(temperature), L.ptr(y), L.ptr(ws), wsb, None,
                                 L.stream_of(x32)), "ThreTopK")
    return y if x.dtype == torch.float32 else y.to(x.dtype)


def dtem_select(k, scores, allowed, tau1=1.0, tau2=30.0, check=True):
    """Soft-k-max block of DTEMBlock._select with the sparse mask
    (dtem.py:1536-1580): scores/allowed [B,Na,K] -> assignment [B,Na,K].
    Differentiable in scores (dtem_select_backward)."""
    if _wants_grad(scores):
        return _DtemSelectFn.apply(scores, allowed, int(k), float(tau1), float(tau2), check)
    return _dtem_select(k, scores, allowed, tau1, tau2, check)


class _DtemSelectFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scores, allowed, k, tau1, tau2, check):
        out = _dtem_select(k, scores, allowed, tau1, tau2, check)
        ctx.save_for_backward(scores, allowed)
        ctx.args = (k, tau1, tau2)
        return out

    @staticmethod
    def backward(ctx, grad_assignment):
        scores, allowed = ctx.saved_tensors
        k, tau1, tau2 = ctx.args
        return dtem_select_backward(k, scores, allowed, grad_assignment, tau1, tau2), None, None, None, None, None


def dtem_select_backward(k, scores, allowed, grad_assignment, tau1=1.0, tau2=30.0):
    """Gradient of the sparse soft-k-max select with respect to its scores,
    as the reference's autograd differentiates dtem.py:1551-1580: through
    the masked row softmax, the logsumexp row energies and ThreTopK over the
    batch's energies (its range included); the over-unity renormalisation
    divides by a detached total.  Rows with no allowed slot and masked slots
    get zero.  Returns grad_scores shaped and typed like scores."""
    dev = L.require_cuda(scores, allowed, grad_assignment)
    s = scores.float().contiguous()
    al = allowed.bool().contiguous()
    g = grad_assignment.float().contiguous()
    bsz, na, kk = s.shape
    out = torch.empty_like(s)
    wsb = L.lib().mn_dtem_select_backward_workspace_bytes(bsz, na)
    ws = torch.empty(int(wsb), dtype=torch.uint8, device=dev)
    L.check(L.lib().mn_dtem_select_backward(bsz, na, kk, L.ptr(s), L.ptr(_as_u8(al)), int(k), float(tau1),
                                            float(tau2), L.ptr(g), L.ptr(out), L.ptr(ws), wsb, None,
                                            L.stream_of(s)), "dtem_select backward")
    return out.to(scores.dtype)


def _dtem_select(k, scores, allowed, tau1, tau2, check):
    dev = L.require_cuda(scores, allowed)
    s = scores.float().contiguous()
    al = allowed.bool().contiguous()
    bsz, na, kk = s.shape
    out = torch.empty_like(s)
    wsb = L.lib().mn_dtem_select_workspace_bytes(bsz, na)
    ws = torch.empty(int(wsb), dtype=torch.uint8, device=dev)
    status = _status(dev)
    L.check(L.lib().mn_dtem_select(bsz, na, kk, L.ptr(s), L.ptr(_as_u8(al)), int(k), float(tau1), float(tau2),
                                   L.ptr(out), L.ptr(ws), wsb, L.ptr(status), L.stream_of(s)), "dtem_select")
    if check:
        _raise_status(status, "dtem_select")
    return out.to(scores.dtype)


# --------------------------------------------------------------------------
# Fused route + gather (canonical eval grouping)
# --------------------------------------------------------------------------
@dataclass
class RouteResult:
    topk_x: torch.Tensor      # [B, k+1, C]  CLS + carriers (centre-of-mass order)
    topk_size: torch.Tensor   # [B, k+1]
    topk_idx: torch.Tensor    # [B, k] int64 patch indices
    size: torch.Tensor        # [B, T]  mass after the last layer
    center: torch.Tensor      # [B, T]  token_center after the last layer
    status: torch.Tensor      # [1] int32 device status word


class RoutePlan:
    """Geometry tables of one (grid, radius, layer budgets), resident on one
    device.  Mirrors the state LocalEncoder keeps in its non-persistent
    buffers and ``_tome_info`` (model.py:336-407)."""

    def __init__(self, grid_size, radius=3.0, r_list=None, device=None, tau1=1.0, tau2=30.0):
        h, w, radius = _check_grid(grid_size, radius)
        lib = L.lib()
        dims = L.RouteDims()
        rc = lib.mn_route_dims_query(h, w, radius, ctypes.byref(dims))
        L.check(rc, "mn_route_dims_query (the fused path needs an even patch count)")
        table = np.zeros(int(dims.table_ints), np.int32)
        L.check(lib.mn_route_tables_fill(h, w, radius, ctypes.byref(dims), table.ctypes.data_as(ctypes.c_void_p)),
                "mn_route_tables_fill")
        self.grid_size = (h, w)
        self.radius = radius
        self.dims = dims
        self.num_patches = h * w
        if r_list is None:
            total = self.num_patches // 2
            r_list = [total // 6] * 6
            r_list[-1] += total - sum(r_list)
        self.r_list = [int(r) for r in r_list]
        for i, r in enumerate(self.r_list):
            r_eff = min(r, self.num_patches // 2)
            if r_eff > dims.valid_rows[i % 2]:
                raise RuntimeError(
                    "DTEM spatial radius leaves fewer eligible donor rows than the required merge budget "
                    f"k={r_eff}; radius={radius}, grid={self.grid_size}")
        self.k = self.num_patches - sum(self.r_list)
        if self.k <= 0 or self.k > self.num_patches:
            self.k = self.num_patches
        self.tau1, self.tau2 = float(tau1), float(tau2)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.table = torch.from_numpy(table).to(self.device)
        self._r_arr = (ctypes.c_int * len(self.r_list))(*self.r_list)

    def workspace_bytes(self, batch):
        return int(L.lib().mn_route_workspace_bytes(ctypes.byref(self.dims), batch, len(self.r_list)))

    def __call__(self, x, metrics, out=None, workspace=None, status=None, check=None):
        """x [B, T, C] (fp32/fp16/bf16), metrics [L, B, T, Cm] -> RouteResult.

        The kernels report data conditions (an infeasible merge budget, an
        empty ThreTopK range, a table error) in the device status word.
        ``check=True`` reads it after the launch and raises (one
        synchronisation), as the reference's budget assert fails closed
        (dtem.py:1536-1546); ``check=False`` leaves ``RouteResult.status`` for
        the caller to read later with ``check_status``.  The default reads it
        unless a CUDA graph is being captured."""
        L.require_cuda(x, metrics)
        if x.device != self.device:
            raise ValueError(f"plan lives on {self.device}, inputs on {x.device}")
        _contig(x, metrics)
        bsz, t, c = x.shape
        nl, mb, mt, cm = metrics.shape
        if t != self.num_patches + 1 or mt != t or mb != bsz or nl != len(self.r_list):
            raise ValueError(f"expected x [B,{self.num_patches + 1},C] and metrics [{len(self.r_list)},B,T,Cm], "
                             f"got {tuple(x.shape)} and {tuple(metrics.shape)}")
        k = self.k
        dev = self.device
        if out is None:
            out = (torch.empty(bsz, k + 1, c, device=dev, dtype=x.dtype),
                   torch.empty(bsz, k + 1, device=dev, dtype=torch.float32),
                   torch.empty(bsz, k, device=dev, dtype=torch.long),
                   torch.empty(bsz, t, device=dev, dtype=torch.float32),
                   torch.empty(bsz, t, device=dev, dtype=torch.float32))
        topk_x, topk_size, topk_idx, size, center = out
        wsb = self.workspace_bytes(bsz)
        if workspace is None:
            workspace = torch.empty(wsb, dtype=torch.uint8, device=dev)
        if status is None:
            status = _status(dev)
        rc = L.lib().mn_route_and_gather(ctypes.byref(self.dims), L.ptr(self.table), bsz, c, cm, nl, self._r_arr, k,
                                         self.tau1, self.tau2, L.ptr(x), L.dtype_code(x.dtype), L.ptr(metrics),
                                         L.dtype_code(metrics.dtype), L.ptr(workspace), wsb, L.ptr(topk_x),
                                         L.ptr(topk_size), L.ptr(topk_idx), L.ptr(size), L.ptr(center),
                                         L.ptr(status), L.stream_of(x))
        L.check(rc, "mn_route_and_gather")
        res = RouteResult(topk_x, topk_size, topk_idx, size, center, status)
        if _default_check(check):
            check_status(res)
        return res


def check_status(result):
    """Raise if the routing call behind ``result`` (a RouteResult, or its
    status tensor) flagged a data condition on the device."""
    status = result.status if isinstance(result, RouteResult) else result
    _raise_status(status, "mn_route_and_gather")


def route_and_gather(x_embed, metrics, grid_size, radius=3.0, r_list=None):
    """One-shot convenience: build a plan and run it."""
    plan = RoutePlan(grid_size, radius, r_list, device=x_embed.device)
    return plan(x_embed, metrics)


# --------------------------------------------------------------------------
# The carrier block's soft-top-k training terms (model.py:1163-1206)
# --------------------------------------------------------------------------
def carrier_ste(topk_x_trace, soft_sel, sorted_topk_indices):
    """The straight-through carrier weights of model.py:1176-1179:
    ``topk_x_trace * (1 + (w - w.detach()))[..., None]`` with
    ``w = soft_sel.gather(1, sorted_topk_indices)``.  The value is
    topk_x_trace; under autograd soft_sel receives, at each carrier's patch,
    the dot product of the carrier's gradient and its features
    (``mn_carrier_ste_backward``) and topk_x_trace the gradient unchanged."""
    if _wants_grad(topk_x_trace, soft_sel):
        return _CarrierSteFn.apply(topk_x_trace, soft_sel, sorted_topk_indices)
    L.require_cuda(topk_x_trace, soft_sel, sorted_topk_indices)
    return topk_x_trace


class _CarrierSteFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, topk_x_trace, soft_sel, sorted_topk_indices):
        L.require_cuda(topk_x_trace, soft_sel, sorted_topk_indices)
        ctx.save_for_backward(topk_x_trace, sorted_topk_indices.long().contiguous())
        ctx.sel_shape, ctx.sel_dtype = soft_sel.shape, soft_sel.dtype
        return topk_x_trace.clone()

    @staticmethod
    def backward(ctx, grad_out):
        x, idx = ctx.saved_tensors
        grad_sel = None
        if ctx.needs_input_grad[1]:
            g = grad_out.to(x.dtype)
            if g.stride(-1) != 1:
                g = g.contiguous()
            xc = x if x.stride(-1) == 1 else x.contiguous()
            bsz, k, c = xc.shape
            n = ctx.sel_shape[1]
            grad_sel = torch.empty(bsz, n, device=x.device, dtype=torch.float32)
            status = _status(x.device)
            L.check(L.lib().mn_carrier_ste_backward(bsz, k, c, L.dtype_code(xc.dtype), L.ptr(xc), xc.stride(0),
                                                    xc.stride(1), L.ptr(g), g.stride(0), g.stride(1), L.ptr(idx), n,
                                                    L.ptr(grad_sel), L.ptr(status), L.stream_of(xc)),
                    "carrier_ste backward")
            if int(status.item()):
                raise ValueError("carrier_ste: carrier patch index out of range")
            grad_sel = grad_sel.to(ctx.sel_dtype)
        return grad_out, grad_sel, None


def soft_topk_aux_repr(x_patches, soft_sel):
    """The soft-top-k auxiliary representation of model.py:1196-1198:
    ``(x_patches * (soft_sel / soft_sel.sum(1, keepdim=True).clamp(min=1e-6))
    [..., None]).sum(1)`` -> float32 [B, C] (``mn_soft_topk_aux``; the
    model's head GEMM on it stays the caller's).  x_patches [B, n, C] may be
    a strided view such as ``x_local[:, 1:]`` (channels contiguous);
    soft_sel [B, n].  Differentiable in both (``mn_soft_topk_aux_backward``)."""
    if _wants_grad(x_patches, soft_sel):
        return _SoftTopkAuxFn.apply(x_patches, soft_sel)
    return _soft_topk_aux(x_patches, soft_sel.float().contiguous())


def _aux_operands(x_patches):
    if x_patches.dim() != 3:
        raise ValueError("x_patches must be [B, n, C]")
    return x_patches if x_patches.stride(-1) == 1 else x_patches.contiguous()


def _soft_topk_aux(x_patches, sel32):
    L.require_cuda(x_patches, sel32)
    x = _aux_operands(x_patches)
    bsz, n, c = x.shape
    if sel32.shape != (bsz, n):
        raise ValueError("soft_sel must be [B, n] for x_patches [B, n, C]")
    aux = torch.empty(bsz, c, device=x.device, dtype=torch.float32)
    L.check(L.lib().mn_soft_topk_aux(bsz, n, c, L.dtype_code(x.dtype), L.ptr(x), x.stride(0), x.stride(1),
                                     L.ptr(sel32), L.ptr(aux), L.stream_of(x)), "soft_topk_aux_repr")
    return aux


class _SoftTopkAuxFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_patches, soft_sel):
        sel32 = soft_sel.float().contiguous()
        ctx.save_for_backward(x_patches, sel32)
        ctx.sel_dtype = soft_sel.dtype
        return _soft_topk_aux(x_patches, sel32)

    @staticmethod
    def backward(ctx, grad_aux):
        x_patches, sel32 = ctx.saved_tensors
        x = _aux_operands(x_patches)
        bsz, n, c = x.shape
        g = grad_aux.float().contiguous()
        grad_x = torch.empty(bsz, n, c, device=x.device, dtype=x.dtype)
        grad_sel = torch.empty(bsz, n, device=x.device, dtype=torch.float32)
        wsb = L.lib().mn_soft_topk_aux_backward_workspace_bytes(bsz, n)
        ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device=x.device)
        L.check(L.lib().mn_soft_topk_aux_backward(bsz, n, c, L.dtype_code(x.dtype), L.ptr(x), x.stride(0), x.stride(1),
                                                  L.ptr(sel32), L.ptr(g), L.ptr(grad_x), L.ptr(grad_sel), L.ptr(ws),
                                                  wsb, L.stream_of(x)), "soft_topk_aux_repr backward")
        return grad_x, grad_sel.to(ctx.sel_dtype)


def carrier_scatter(topk_x, topk_idx, num_patches):
    """Transpose of the carrier gather: [B, k+1, C] -> [B, P, C], carrier i at
    patch topk_idx[b, i], zeros elsewhere."""
    dev = L.require_cuda(topk_x, topk_idx)
    topk_x = topk_x.contiguous()
    idx = topk_idx.long().contiguous()
    bsz, k1, c = topk_x.shape
    out = torch.empty(bsz, num_patches, c, device=dev, dtype=topk_x.dtype)
    L.check(L.lib().mn_carrier_scatter(bsz, k1 - 1, num_patches, c, L.dtype_code(topk_x.dtype), L.ptr(topk_x),
                                       L.ptr(idx), L.ptr(out), L.stream_of(topk_x)), "carrier_scatter")
    return out
