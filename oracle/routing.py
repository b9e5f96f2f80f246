"""numpy restatement of MergeNet's DTEM spatial routing (the oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Every function computes in float32 where the reference computes in float32,
and follows the reference's operation order where it is observable in the last
bits (normalise-then-dot, ``logsumexp(...).exp()``, the global ThreTopK range,
sequential scatter-add order).  Reference files are cited relative to the
MergeNet project root.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
EPS32 = np.finfo(np.float32).eps


# --------------------------------------------------------------------------
# Geometry  (opentome/timm/dtem.py:50-127)
# --------------------------------------------------------------------------
def build_patch_spatial_adjacency(grid_size, radius):
    """Boolean [P,P] matrix of patch pairs whose squared grid distance <= R^2.

    Follows opentome/timm/dtem.py:50-92: row-major patches, squared Euclidean
    distance compared in float32 against ``radius * radius``.
    """
    if not isinstance(grid_size, (tuple, list)) or len(grid_size) != 2:
        raise ValueError(f"grid_size must be a (height, width) pair, got {grid_size!r}")
    if any(isinstance(v, bool) or not isinstance(v, (int, np.integer)) for v in grid_size):
        raise ValueError(f"grid_size values must be integers, got {grid_size!r}")
    h, w = int(grid_size[0]), int(grid_size[1])
    if h <= 0 or w <= 0:
        raise ValueError(f"grid_size values must be positive, got {(h, w)!r}")
    if isinstance(radius, bool):
        raise ValueError("radius must be a positive finite number, not bool")
    radius = float(radius)
    if not math.isfinite(radius) or radius <= 0:
        raise ValueError(f"radius must be a positive finite number, got {radius!r}")
    idx = np.arange(h * w, dtype=np.int64)
    rows, cols = idx // w, idx % w
    d2 = (rows[:, None] - rows[None, :]) ** 2 + (cols[:, None] - cols[None, :]) ** 2
    return d2.astype(F32) <= F32(radius * radius)


def adjacency_to_padded_neighbors(adjacency):
    """[P,K] neighbour table in ascending patch order (dtem.py:95-127).

    Padding entries hold index 0 and validity False.
    """
    adjacency = np.asarray(adjacency)
    if adjacency.ndim != 2 or adjacency.shape[0] != adjacency.shape[1] or adjacency.shape[0] == 0:
        raise ValueError("adjacency must be non-empty and square")
    if adjacency.dtype != np.bool_:
        raise ValueError("adjacency must have bool dtype")
    counts = adjacency.sum(axis=-1)
    kmax = int(counts.max())
    if kmax <= 0:
        raise ValueError("every patch must have at least one spatial neighbor")
    p = adjacency.shape[0]
    indices = np.zeros((p, kmax), dtype=np.int64)
    valid = np.zeros((p, kmax), dtype=np.bool_)
    for row in range(p):
        cols = np.nonzero(adjacency[row])[0]
        indices[row, : cols.size] = cols
        valid[row, : cols.size] = True
    return indices, valid


def parse_r(num_layers, r, total=None):
    """Per-layer merge budget schedule (opentome/tome/tome.py:12-53)."""
    inflect = 0
    if isinstance(r, list):
        if len(r) < num_layers:
            r = r + [0] * (num_layers - len(r))
        return list(r)
    if isinstance(r, tuple):
        r, inflect = r
    min_val = int(r * (1.0 - inflect))
    max_val = 2 * r - min_val
    if num_layers <= 1:
        r_list = [int(r)] * num_layers
    else:
        step = (max_val - min_val) / (num_layers - 1)
        r_list = [int(min_val + step * i) for i in range(num_layers)]
    if total is not None:
        remainder = total - sum(r_list)
        if remainder != 0:
            if inflect < 0:
                r_list[0] += remainder
            else:
                r_list[-1] += remainder
    return r_list


# --------------------------------------------------------------------------
# Scoring  (dtem.py:219-234 mapping, :748-761 dot)
# --------------------------------------------------------------------------
def map_sorted_receivers(nbr_idx, nbr_valid, donor_patch, receiver_patch):
    """Static neighbour -> receiver slot through a sorted receiver list.

    Mirrors ``gather_patch_spatial_neighbors(..., receivers_are_sorted=True)``
    (dtem.py:219-234): left insertion point clamped to Nb-1, valid only where
    the static slot is valid and the receiver patch really is that neighbour.
    """
    nbr_idx = np.asarray(nbr_idx)
    donor_patch = np.asarray(donor_patch, dtype=np.int64)
    receiver_patch = np.asarray(receiver_patch, dtype=np.int64)
    b, na = donor_patch.shape
    nb = receiver_patch.shape[1]
    pn = nbr_idx[donor_patch]  # [B,Na,K]
    sv = np.asarray(nbr_valid)[donor_patch]
    pos = np.empty_like(pn)
    for i in range(b):
        pos[i] = np.searchsorted(receiver_patch[i], pn[i], side="left")
    safe = np.minimum(pos, nb - 1)
    found = np.take_along_axis(receiver_patch, safe.reshape(b, -1), axis=1).reshape(pn.shape) == pn
    valid = sv & (pos < nb) & found
    return safe, valid


def sparse_spatial_score(a, b, nbr_idx, nbr_valid, donor_patch, receiver_patch):
    """(scores, receiver_indices, receiver_valid) of dtem.py:813-848 (CPU path :749-761)."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    ridx, rvalid = map_sorted_receivers(nbr_idx, nbr_valid, donor_patch, receiver_patch)
    bidx = np.arange(a.shape[0])[:, None, None]
    cand = b[bidx, ridx]  # [B,Na,K,C]
    scores = (a[:, :, None, :] * cand).sum(axis=-1, dtype=F32)
    scores = (scores * rvalid.astype(F32)).astype(F32)
    return scores, ridx, rvalid


def sparse_neighbor_dot(a, b, receiver_indices, receiver_valid):
    """Indexed dot of dtem.py:680-687 (CPU path :626-629)."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    bidx = np.arange(a.shape[0])[:, None, None]
    cand = b[bidx, receiver_indices]
    s = (a[:, :, None, :] * cand).sum(axis=-1, dtype=F32)
    return (s * np.asarray(receiver_valid).astype(F32)).astype(F32)


def sparse_neighbor_dot_backward(a, b, receiver_indices, receiver_valid, grad_scores):
    """Gradients of sparse_neighbor_dot (the torch path of
    _SparseNeighborDot.backward, dtem.py:667-676): grad_a[d] = sum_k g[d,k]
    b[r(d,k)]; grad_b[s] += g[d,k] a[d] scatter-added over the flattened
    donor-major edge list (np.add.at applies the edges in that order)."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    ridx = np.asarray(receiver_indices)
    g = (np.asarray(grad_scores, dtype=F32) * np.asarray(receiver_valid).astype(F32)).astype(F32)
    bidx = np.arange(a.shape[0])[:, None, None]
    grad_a = (g[..., None] * b[bidx, ridx]).sum(axis=2, dtype=F32).astype(F32)
    grad_b = np.zeros_like(b)
    contrib = (g[..., None] * a[:, :, None, :]).astype(F32)
    for i in range(a.shape[0]):
        np.add.at(grad_b[i], ridx[i].reshape(-1), contrib[i].reshape(-1, a.shape[-1]))
    return grad_a, grad_b


def sparse_weighted_transport(assignment, values, receiver_indices, receiver_valid, num_receivers):
    """out[b,s,:] = sum over (d,k) with slot s of assignment*values, in (d,k) order.

    Restates the torch fallback of dtem.py:911-926 (a sequential scatter-add
    over the flattened donor-major edge list).
    """
    assignment = np.asarray(assignment, dtype=F32)
    values = np.asarray(values, dtype=F32)
    ridx = np.asarray(receiver_indices)
    rvalid = np.asarray(receiver_valid)
    bsz, na, k = assignment.shape
    c = values.shape[-1]
    out = np.zeros((bsz, num_receivers, c), dtype=F32)
    contrib = (assignment[..., None] * values[:, :, None, :]).astype(F32)
    contrib = (contrib * rvalid[..., None].astype(F32)).astype(F32)
    for i in range(bsz):
        np.add.at(out[i], ridx[i].reshape(-1), contrib[i].reshape(-1, c))
    return out


# --------------------------------------------------------------------------
# ThreTopK  (opentome/utils/thetopk.py:4-43)
# --------------------------------------------------------------------------
def _logcumsumexp_rows(x):
    """Row-wise inclusive log-cum-sum-exp, accumulated in float64 and rounded
    to float32 per output, as the CPU ATen kernel does (double accumulator,
    ``log1p(exp(min - max)) + max`` combine step)."""
    x64 = x.astype(np.float64)
    out = np.empty_like(x, dtype=F32)
    cum = np.full(x.shape[0], -np.inf)
    with np.errstate(invalid="ignore", over="ignore"):
        for j in range(x.shape[1]):
            v = x64[:, j]
            mn = np.minimum(v, cum)
            mx = np.maximum(v, cum)
            take = (mn != mx) | np.isfinite(mn)
            comb = np.log1p(np.exp(mn - mx)) + mx
            cum = np.where(take, comb, v)
            out[:, j] = cum.astype(F32)
    return out


def thre_topk(x, k, temperature=30.0):
    """Threshold soft top-k with ONE global range over the whole input."""
    x = np.asarray(x, dtype=F32)
    if x.ndim == 1:
        x = x[None]
    x_range = F32(x.max() - x.min())
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        x = ((x / x_range).astype(F32) * F32(temperature)).astype(F32)
        n = x.shape[1]
        xs = np.sort(x, axis=-1)
        lse1 = _logcumsumexp_rows(xs)
        lse2_cum = _logcumsumexp_rows(-xs[:, ::-1])[:, ::-1]
        lse2 = np.concatenate([lse2_cum[:, 1:], np.full((x.shape[0], 1), -np.inf, F32)], axis=1)
        m = np.arange(n - 1, -1, -1, dtype=np.int64)[None, :]
        k_m = (k - m).astype(np.int64)
        log_exp_sum = (lse1 + lse2).astype(F32)
        term = (np.sqrt((k_m * k_m).astype(F32) + np.exp(log_exp_sum)).astype(F32) + k_m.astype(F32)).astype(F32)
        x_lamb = (lse1 - np.log((np.abs(term) + F32(1e-8)).astype(F32))).astype(F32)
        shift = np.concatenate([xs[:, 1:], np.full((x.shape[0], 1), np.inf, F32)], axis=1)
        mask = (x_lamb >= xs) & (x_lamb <= shift)
        idx = np.argmax(mask, axis=-1)
        lamb = np.take_along_axis(x_lamb, idx[:, None], axis=-1)
        delta = (x - lamb).astype(F32)
        y = np.where(delta > 0,
                     (F32(1.0) - (F32(0.5) * np.exp(-delta)).astype(F32)).astype(F32),
                     (F32(0.5) * np.exp(delta)).astype(F32))
    return y.astype(F32)


# --------------------------------------------------------------------------
# Select  (dtem.py:1464-1580, soft-k-max branch with the sparse spatial mask)
# --------------------------------------------------------------------------

def thre_topk_backward(x, k, grad_y, temperature=30.0):
    """Gradient of ThreTopK with respect to x, in float64: the closed form of
    what the reference's autograd computes through thetopk.py:4-43.  With
    x~ = x / R * T (R = max - min over the whole input), b the row's bracket
    and lambda = lse1[b] - log(|term[b]| + 1e-8):
    dx~_i = f'(d_i) g_i + [s(i) <= b] dlse1 e^{x~_i - lse1[b]}
            - [s(i) > b] dL e^{-x~_i - lse2[b]},
    with dlambda = -sum_i f'(d_i) g_i, dL = d|term|/dL * (-dlambda / (|term| + 1e-8)),
    dlse1 = dlambda + dL; then dx = dx~ T / R, and dR = -sum dx~_i x_i T / R^2
    goes to the maximum (+) and minimum (-) elements, split evenly over ties.
    s(i) is i's position in the row's stable ascending sort."""
    x = np.asarray(x, np.float64)
    g = np.asarray(grad_y, np.float64)
    squeeze = x.ndim == 1
    if squeeze:
        x, g = x[None], g[None]
    r_range = x.max() - x.min()
    xt = x / r_range * temperature
    rows, n = x.shape
    dxt = np.zeros_like(xt)
    for r in range(rows):
        perm = np.argsort(xt[r], kind="stable")
        xs = xt[r, perm]
        lse1 = xs[-1] + np.log(np.cumsum(np.exp(xs - xs[-1])))
        suffix = np.cumsum(np.exp(xs[0] - xs)[::-1])[::-1]
        lse2 = np.concatenate([-xs[0] + np.log(suffix[1:]), [-np.inf]])
        km = k - (n - 1 - np.arange(n))
        big_l = lse1 + lse2
        term = np.sqrt(km * km + np.exp(big_l)) + km
        xl = lse1 - np.log(np.abs(term) + 1e-8)
        mask = (xl >= xs) & (xl <= np.concatenate([xs[1:], [np.inf]]))
        b = int(np.argmax(mask)) if mask.any() else 0
        d = xt[r] - xl[b]
        dd = g[r] * np.where(d > 0, 0.5 * np.exp(-d), 0.5 * np.exp(d))
        dlam = -dd.sum()
        el = np.exp(big_l[b])
        dl = -dlam / (np.abs(term[b]) + 1e-8) * np.sign(term[b]) * 0.5 / np.sqrt(km[b] ** 2 + el) * el
        dxs = np.zeros(n)
        dxs[:b + 1] = (dlam + dl) * np.exp(xs[:b + 1] - lse1[b])
        if b < n - 1:
            dxs[b + 1:] = -dl * np.exp(-xs[b + 1:] - lse2[b])
        dxt[r] = dd
        dxt[r, perm] += dxs
    dx = dxt * temperature / r_range
    d_range = (dxt * (-x * temperature / r_range ** 2)).sum()
    is_max, is_min = x == x.max(), x == x.min()
    dx[is_max] += d_range / is_max.sum()
    dx[is_min] -= d_range / is_min.sum()
    return dx[0] if squeeze else dx

def select_backward(k, scores, allowed, grad_assign, tau1=1.0, tau2=30.0):
    """Gradient of the sparse soft-k-max select (dtem.py:1551-1580) with
    respect to its scores, in float64, as the reference's autograd takes it.
    Per valid donor row (any allowed slot), with p the masked softmax of
    scores / tau1, E = exp(logsumexp), y = ThreTopK(E over the batch) and
    t = max(sum_j p_j y - 1, 0) + 1 (detached):
      dp_j = G_j y / t,   dy = sum_j G_j p_j / t,
      dE = thre_topk_backward(E, k, dy) (invalid rows: E = 0, no gradient),
      dscores_j = p_j (dp_j - sum_l dp_l p_l + dE E) / tau1 on allowed slots."""
    s = np.asarray(scores, np.float64)
    al = np.asarray(allowed, np.bool_)
    g = np.asarray(grad_assign, np.float64)
    valid = al.any(-1)
    logits = np.where(al, s / tau1, -np.inf)
    m = np.where(valid, logits.max(-1), 0.0)
    e = np.where(al, np.exp(logits - m[..., None]), 0.0)
    tot = np.where(valid, e.sum(-1), 1.0)
    p = e / tot[..., None]
    energy = np.where(valid, np.exp(np.log(tot) + m), 0.0)
    y = thre_topk(energy.astype(F32), k, tau2).astype(np.float64).reshape(energy.shape) * valid
    t = np.maximum((p * y[..., None]).sum(-1) - 1.0, 0.0) + 1.0
    gt = g / t[..., None]
    dp = gt * y[..., None]
    dy = (gt * p).sum(-1) * valid
    de = thre_topk_backward(energy, k, dy, tau2).reshape(energy.shape) * valid
    inner = (dp * p).sum(-1)
    ds = p * (dp - inner[..., None] + (de * energy)[..., None]) / tau1
    return np.where(al & valid[..., None], ds, 0.0)


def _softmax_lastdim(x):
    """exp(x - max) * (1 / sum) like the CPU softmax kernel."""
    mx = x.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp((x - mx).astype(F32)).astype(F32)
    s = e.sum(axis=-1, keepdims=True, dtype=F32)
    return (e * (F32(1.0) / s).astype(F32)).astype(F32)


def _logsumexp_lastdim(x):
    """log(sum(exp(x - m))) + m with m zeroed where infinite (ATen logsumexp)."""
    m = x.max(axis=-1, keepdims=True)
    m = np.where(np.abs(m) == np.inf, F32(0), m).astype(F32)
    with np.errstate(invalid="ignore", divide="ignore"):
        s = np.exp((x - m).astype(F32)).astype(F32).sum(axis=-1, dtype=F32)
        return (np.log(s).astype(F32) + m[..., 0]).astype(F32)


class InfeasibleBudget(RuntimeError):
    """Fewer donor rows with a legal receiver than the merge budget k."""


def select(k, scores, allowed, tau1=1.0, tau2=30.0):
    """Sparse-mask soft-k-max assignment [B,Na,K] from scores [B,Na,K]."""
    scores = np.asarray(scores, dtype=F32)
    allowed = np.asarray(allowed, dtype=np.bool_)
    valid_row = allowed.any(axis=-1)
    if not bool((valid_row.sum(axis=-1) >= int(k)).all()):
        raise InfeasibleBudget(
            "DTEM spatial radius leaves fewer eligible donor rows than the "
            f"required merge budget k={int(k)}")
    logits = (scores / F32(tau1)).astype(F32)
    logits = np.where(allowed, logits, F32(-np.inf)).astype(F32)
    safe = np.where(valid_row[..., None], logits, F32(0)).astype(F32)
    with np.errstate(over="ignore"):
        energy = np.exp(_logsumexp_lastdim(safe)).astype(F32)
    energy = np.where(valid_row, energy, F32(0)).astype(F32)
    row_khot = (thre_topk(energy, k, tau2) * valid_row.astype(F32)).astype(F32)
    prob = (_softmax_lastdim(safe) * allowed.astype(F32)).astype(F32)
    khot = (prob * row_khot[..., None]).astype(F32)
    tmp = (np.maximum(khot.sum(axis=-1, keepdims=True, dtype=F32) - F32(1), F32(0)) + F32(1)).astype(F32)
    return (khot / tmp).astype(F32), energy, row_khot


# --------------------------------------------------------------------------
# One merge layer, alternating_per_layer_fast grouping (dtem.py:1687-2223)
# --------------------------------------------------------------------------
class Geometry:
    """Static tables for one (grid, radius): the [P,K] neighbour table."""

    def __init__(self, grid_size, radius=3.0):
        self.grid_size = (int(grid_size[0]), int(grid_size[1]))
        self.radius = float(radius)
        self.adjacency = build_patch_spatial_adjacency(self.grid_size, self.radius)
        self.nbr_idx, self.nbr_valid = adjacency_to_padded_neighbors(self.adjacency)
        self.num_patches = self.grid_size[0] * self.grid_size[1]


def normalize_metric(metric):
    """metric / max(||metric||, 1e-6) in float32 (dtem.py:1689-1691)."""
    m = np.asarray(metric).astype(F32)
    norm = np.sqrt((m * m).sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)
    norm = np.maximum(norm, F32(1e-6))
    return (m / norm).astype(F32)


def merge_layer(x, size, center, metric, r, layer_index, geom, tau1=1.0, tau2=30.0):
    """One eval-mode soft-merge layer with a CLS prefix.

    x [B,T,C] float32, size [B,T] float32, center [B,T] float32 (or None at the
    first layer), metric [B,T,Cm].  Returns (x_out, size_out, center_out, info).
    """
    x = np.asarray(x, dtype=F32)
    size = np.asarray(size, dtype=F32)
    bsz, t, c = x.shape
    m = normalize_metric(metric)
    n = t
    r = min(int(r), (n - 1) // 2)
    if center is None:
        center_in = np.broadcast_to(np.arange(t, dtype=F32), (bsz, t)).copy()
        cls_center = np.zeros((bsz, 1), F32)
    else:
        center_in = np.asarray(center, dtype=F32)
        cls_center = center_in[:, :1].copy()
    if r <= 0:
        return x, size, center_in, None
    n_tokens = n - 1
    assert n_tokens % 2 == 0, "alternating_per_layer_fast needs an even patch count"
    dp = 0 if layer_index % 2 else 1  # donor patch parity (dtem.py:1812)
    rp = 1 - dp
    dsl = slice(1 + dp, n, 2)
    rsl = slice(1 + rp, n, 2)
    xa, xb = x[:, dsl], x[:, rsl]
    a, b = m[:, dsl], m[:, rsl]
    wa, wb = size[:, dsl], size[:, rsl]
    ca, cb = center_in[:, dsl], center_in[:, rsl]
    na, nb = xa.shape[1], xb.shape[1]
    donor_patch = np.broadcast_to(np.arange(dp, n_tokens, 2), (bsz, na))
    receiver_patch = np.broadcast_to(np.arange(rp, n_tokens, 2), (bsz, nb))
    scores, ridx, rvalid = sparse_spatial_score(a, b, geom.nbr_idx, geom.nbr_valid, donor_patch, receiver_patch)
    assign, energy, row_khot = select(r, scores, rvalid, tau1, tau2)
    weighted_xa = (wa[..., None] * xa).astype(F32)
    xb_contrib = sparse_weighted_transport(assign, weighted_xa, ridx, rvalid, nb)
    wb_contrib = sparse_weighted_transport(assign, wa[..., None], ridx, rvalid, nb)[..., 0]
    xb_new = ((wb[..., None] * xb).astype(F32) + xb_contrib).astype(F32)
    wb_new = (wb + wb_contrib).astype(F32)
    tmp = (F32(1) - assign.sum(axis=-1, dtype=F32)).astype(F32)
    wa_new = (wa * np.clip(tmp, F32(0), F32(1))).astype(F32)
    wb_safe = np.maximum(wb_new, EPS32).astype(F32)
    xb_new = (xb_new / wb_safe[..., None]).astype(F32)
    cc = np.zeros((bsz, nb), F32)
    contrib = (assign * (wa * ca).astype(F32)[..., None]).astype(F32)
    for i in range(bsz):
        np.add.at(cc[i], ridx[i].reshape(-1), contrib[i].reshape(-1))
    cb_new = (((wb * cb).astype(F32) + cc).astype(F32) / wb_safe).astype(F32)
    x_out = np.empty_like(x)
    size_out = np.empty_like(size)
    center_out = np.empty((bsz, t), F32)
    x_out[:, 0] = x[:, 0]
    size_out[:, 0] = size[:, 0]
    center_out[:, :1] = cls_center
    x_out[:, dsl], x_out[:, rsl] = xa, xb_new
    size_out[:, dsl], size_out[:, rsl] = wa_new, wb_new
    center_out[:, dsl], center_out[:, rsl] = ca, cb_new
    info = dict(scores=scores, receiver_indices=ridx, receiver_valid=rvalid,
                assign=assign, energy=energy, row_khot=row_khot)
    return x_out, size_out, center_out, info


def select_carriers(size, center, k):
    """Exact top-k by mass, then ascending centre of mass (model.py:1157-1183).

    Ties in mass keep the lower patch index; ties in centre keep the lower
    patch index (``torch.topk(sorted=False)`` and the unstable ``argsort``
    leave both unspecified).
    """
    strength = np.asarray(size, dtype=F32)[:, 1:]
    com = np.asarray(center, dtype=F32)[:, 1:]
    bsz, p = strength.shape
    out = np.empty((bsz, k), np.int64)
    for i in range(bsz):
        order = np.lexsort((np.arange(p), -strength[i].astype(np.float64)))
        top = order[:k]
        top = top[np.lexsort((top, com[i][top].astype(np.float64)))]
        out[i] = top
    return out


def route_and_gather(x, metrics, r_list, geom, tau1=1.0, tau2=30.0, keep_info=False):
    """Six merge layers + carrier gather of the canonical model.

    Returns dict(topk_x [B,k+1,C], topk_size [B,k+1], topk_idx [B,k] (patch
    indices), size [B,T], center [B,T], x_local [B,T,C]).  Follows
    model.py:574-590 then model.py:1157-1183.
    """
    x = np.asarray(x, dtype=F32)
    bsz, t, _ = x.shape
    size = np.ones((bsz, t), F32)
    center = None
    infos = []
    for i, r in enumerate(r_list):
        x, size, center, info = merge_layer(x, size, center, metrics[i], r, i, geom, tau1, tau2)
        if keep_info:
            infos.append(info)
    p = t - 1
    k = t - sum(r_list) - 1
    if k <= 0 or k > p:
        k = p
    idx = select_carriers(size, center, k)
    full = idx + 1
    bi = np.arange(bsz)[:, None]
    topk_x = np.concatenate([x[:, :1], x[bi, full]], axis=1)
    topk_size = np.concatenate([size[:, :1], size[bi, full]], axis=1)
    out = dict(topk_x=topk_x, topk_size=topk_size, topk_idx=idx, size=size,
               center=center, x_local=x)
    if keep_info:
        out["layers"] = infos
    return out


def carrier_margin(size, k):
    """Per-image gap between the k-th and (k+1)-th largest patch mass, as a
    fraction of the k-th: the room a carrier set has against rounding."""
    s = -np.sort(-np.asarray(size, dtype=np.float64)[:, 1:], axis=1)
    return (s[:, k - 1] - s[:, k]) / np.abs(s[:, k - 1])
