"""Module-level drop-in for the merge half of the reference's DTEMBlock.

``DTEMMergeBlock`` keeps the two methods LocalEncoder.forward calls on its
merge block (opentome/models/mergenet/model.py:574-590) with the reference's
signatures, return values and ``_tome_info`` side effects:

* ``_select(k, a, b, a_orig_idx, b_orig_idx) -> (assign, None)``
  (opentome/timm/dtem.py:1464-1580): sparse spatial scores, the budget check
  and the soft-k-max assignment; sets ``assign_layout = "spatial_sparse"``,
  ``assign_b_indices`` and ``assign_valid_mask``.
* ``_merge_train(x, size, r, n, {"metric": m}, source_matrix) ->
  (x, size, n, None, None)`` (dtem.py:1687-2223; the normalised metric when
  the layer merges nothing): metric normalisation,
  donor/receiver grouping, the transport of features and mass, the mass
  update, centre-of-mass tracking (``token_center``) and the row-major
  restore.

The scoring, the select block and both transports run on the library's CUDA
kernels (``sparse_spatial_score``, ``dtem_select``,
``sparse_weighted_transport``); the remaining elementwise steps are PyTorch
on the same device.  It covers the configuration the canonical model uses:
global candidates with a 2-D spatial radius on the sparse backend, soft-k-max
selection, and ``source_trace_mode`` "center" or "none", in eval mode and in
training mode.  Training is differentiable end to end in x, size and the
metric: the score, select and transport kernels have CUDA backward passes,
and the donors' mass update keeps the reference's straight-through form
``wa * (tmp + (clamp(tmp, 0, 1) - tmp).detach())``.  Training groups tokens
as the reference does (dtem.py:1755-1800): ``train_grouping``
"random_per_sample" (the default) draws ``torch.rand(B, n - 1)`` on the
tokens' device and splits its argsort; the deterministic modes use
``build_eval_group_indices`` with ``train_grouping_seed``.  Other
configurations (flat windows, the dense backend, dense source matrices)
raise ``NotImplementedError`` before any device work.  For the whole
six-layer inference loop plus the carrier block in a handful of launches,
use ``RoutePlan`` instead.
"""
from __future__ import annotations

import torch

from .routing import (
    build_patch_spatial_adjacency,
    build_patch_spatial_neighbors,
    dtem_select,
    sparse_spatial_score,
    sparse_weighted_transport,
    sparse_weighted_transport_pair,
)

EVAL_GROUPINGS = ("alternating", "alternating_per_layer", "alternating_per_layer_fast", "seeded")


def build_eval_group_indices(n_tokens, batch_size, device, mode="alternating_per_layer", seed=0, layer_index=0):
    """Donor / receiver token positions of one merge layer
    (build_dtem_eval_group_indices, dtem.py:1125-1188): [B, n/2] each."""
    n_tokens, batch_size, layer_index = int(n_tokens), int(batch_size), int(layer_index)
    if n_tokens < 0:
        raise ValueError(f"n_tokens must be non-negative, got {n_tokens}")
    if batch_size <= 0:
        raise ValueError(f"batch_size must be positive, got {batch_size}")
    if mode not in EVAL_GROUPINGS:
        raise ValueError(f"Unsupported DTEM eval grouping {mode!r}; expected one of {EVAL_GROUPINGS}")
    base = torch.arange(n_tokens, device=device, dtype=torch.long)
    if mode == "alternating":
        perm = torch.cat([base[1::2], base[0::2]])
    elif mode in ("alternating_per_layer", "alternating_per_layer_fast"):
        perm = torch.cat([base[0::2], base[1::2]]) if layer_index % 2 else torch.cat([base[1::2], base[0::2]])
    else:
        gen = torch.Generator(device="cpu")
        gen.manual_seed((int(seed) + 1_000_003 * layer_index) % (2**63 - 1))
        perm = torch.randperm(n_tokens, generator=gen, device="cpu").to(device)
    nd = n_tokens // 2
    return perm[:nd].unsqueeze(0).expand(batch_size, -1), perm[nd:].unsqueeze(0).expand(batch_size, -1)


def default_tome_info(grid_size, radius=3.0, metric="euclidean", device=None, eval_grouping="alternating_per_layer_fast",
                      tau1=1.0, tau2=30.0, num_prefix_tokens=1):
    """The ``_tome_info`` keys the merge path reads, filled the way
    LocalEncoder fills them for a spatial-radius model (model.py:336-405,
    :552-567), with the neighbour tables built by the library."""
    nbr, valid = build_patch_spatial_neighbors(grid_size, radius, metric, device=device)
    return {
        "window_size": 0,
        "dtem_spatial_radius": float(radius),
        "dtem_spatial_metric": metric,
        "dtem_spatial_backend": "sparse",
        "patch_grid_size": tuple(int(v) for v in grid_size),
        "num_prefix_tokens": int(num_prefix_tokens),
        "spatial_adjacency": None,
        "spatial_neighbor_indices": nbr,
        "spatial_neighbor_valid": valid,
        "tau1": float(tau1),
        "tau2": float(tau2),
        "use_softkmax": True,
        "class_token": num_prefix_tokens > 0,
        "source_trace_mode": "center",
        "eval_grouping": eval_grouping,
        "eval_grouping_seed": 0,
        "merge_layer_index": 0,
        "t": 1,
        "token_center": None,
    }


class DTEMMergeBlock(torch.nn.Module):
    """The merge block LocalEncoder calls (DTEMMergeOnly, model.py:224-230),
    on the library's kernels.  It has no parameters; ``_tome_info`` is shared
    with the caller exactly as the reference shares it."""

    def __init__(self, tome_info=None):
        super().__init__()
        self._tome_info = tome_info if tome_info is not None else {}

    # ------------------------------------------------------------- checks
    def _check_supported(self):
        info = self._tome_info
        window = info.get("window_size")
        if window is not None and window > 0:
            raise NotImplementedError("flat-window DTEM candidates are not on the B200 path")
        if info.get("dtem_spatial_radius") is None:
            raise NotImplementedError("global DTEM candidates without a spatial radius are not on the B200 path")
        backend = info.get("dtem_spatial_backend", "dense")
        if backend != "sparse":
            raise NotImplementedError(f"dtem_spatial_backend {backend!r}: the B200 path is the sparse backend")
        if info.get("use_softkmax") is False:
            raise NotImplementedError("the sorted-softmax (use_softkmax=False) select is not on the B200 path")
        mode = info.get("source_trace_mode", "none")
        if mode not in ("center", "none"):
            raise NotImplementedError(f"source_trace_mode {mode!r} (dense source matrices) is not on the B200 path")

    # ------------------------------------------------------------- select
    def _select(self, k, a, b, a_orig_idx=None, b_orig_idx=None):
        """(B, Na, K) soft-k-max assignment over the sparse spatial
        neighbourhoods (dtem.py:1464-1580); returns (assign, None)."""
        self._check_supported()
        info = self._tome_info
        if a_orig_idx is None or b_orig_idx is None:
            raise RuntimeError("DTEM spatial masking requires absolute donor/receiver token indices")
        nbr, valid = info.get("spatial_neighbor_indices"), info.get("spatial_neighbor_valid")
        if nbr is None or valid is None:
            raise RuntimeError("sparse DTEM spatial scoring is enabled but the neighbor table is unavailable")
        prefix = info.get("num_prefix_tokens", 1)
        scores, receiver_indices, allowed = sparse_spatial_score(
            a, b, nbr, valid, a_orig_idx.long() - prefix, b_orig_idx.long() - prefix)
        info["assign_layout"] = "spatial_sparse"
        info["assign_b_indices"] = receiver_indices
        info["assign_valid_mask"] = allowed
        try:
            assign = dtem_select(int(k), scores, allowed, info.get("tau1", 1.0), info["tau2"])
        except RuntimeError as exc:
            if "merge budget" not in str(exc):
                raise
            raise RuntimeError(
                "DTEM spatial radius leaves fewer eligible donor rows than the required merge budget "
                f"k={int(k)}; radius={info.get('dtem_spatial_radius')}, grid={info.get('patch_grid_size')}") from exc
        return assign.to(scores.dtype), None

    # -------------------------------------------------------------- merge
    def _groups(self, n_tokens, bsz, dev):
        """Donor / receiver positions (before the prefix offset) and whether
        they are the strided parity split (dtem.py:1755-1812)."""
        info = self._tome_info
        layer = info.get("merge_layer_index", 0)
        if self.training:
            grouping = info.get("train_grouping", "random_per_sample")
            if grouping == "random_per_sample":
                perm = torch.argsort(torch.rand(bsz, n_tokens, device=dev), dim=1)
                nd = n_tokens // 2
                return perm[:, :nd], perm[:, nd:], False
            seed = info.get("train_grouping_seed", 0)
        else:
            grouping = info.get("eval_grouping", "alternating_per_layer")
            seed = info.get("eval_grouping_seed", 0)
        a_idx, b_idx = build_eval_group_indices(n_tokens, bsz, dev, grouping, seed, layer)
        return a_idx, b_idx, grouping == "alternating_per_layer_fast" and n_tokens % 2 == 0

    def _merge_train(self, x, size, r, n, metric, source_matrix=None):
        """One soft merge layer (dtem.py:1687-2223); differentiable when
        autograd records it, with the centre tracking outside the graph."""
        self._check_supported()
        info = self._tome_info
        m = metric["metric"].float()
        m = m / m.norm(dim=-1, keepdim=True).clamp_min(1e-6)
        r = min(r, (n - 1) // 2)
        if r <= 0:
            return x, size, n, m, None
        if size is not None and size.ndim == 2:
            size = size.unsqueeze(-1)
        trace_center = info.get("source_trace_mode", "none") == "center"
        bsz, t_tokens, c = x.shape
        dev = x.device
        offset = 1 if info.get("class_token", True) else 0
        n_tokens = n - offset
        layer = info.get("merge_layer_index", 0)
        a_idx, b_idx, strided = self._groups(n_tokens, bsz, dev)
        a_idx, b_idx = a_idx + offset, b_idx + offset
        if strided:
            donor_parity = 0 if layer % 2 else 1
            ds = slice(offset + donor_parity, offset + n_tokens, 2)
            rs = slice(offset + 1 - donor_parity, offset + n_tokens, 2)
            a_sorted, b_sorted = a_idx, b_idx
            xa, xb = x[:, ds].float(), x[:, rs].float()
            a, b = m[:, ds].contiguous(), m[:, rs].contiguous()
            wa, wb = size[:, ds, 0].float(), size[:, rs, 0].float()
        else:
            a_sorted, _ = torch.sort(a_idx, dim=1)
            b_sorted, _ = torch.sort(b_idx, dim=1)
            gather = lambda t, idx: torch.gather(t, 1, idx.unsqueeze(-1).expand(-1, -1, t.shape[-1]))  # noqa: E731
            xa, xb = gather(x, a_sorted).float(), gather(x, b_sorted).float()
            a, b = gather(m, a_sorted).contiguous(), gather(m, b_sorted).contiguous()
            wa = torch.gather(size[..., 0], 1, a_sorted).float()
            wb = torch.gather(size[..., 0], 1, b_sorted).float()
        wa0, wb0 = wa.detach().clone(), wb.detach().clone()
        if trace_center:
            tc = info.get("token_center")
            if tc is None:
                tc = torch.arange(t_tokens, device=dev, dtype=torch.float32).unsqueeze(0).expand(bsz, -1)
            ca = tc[:, ds] if strided else torch.gather(tc, 1, a_sorted)
            cb = tc[:, rs] if strided else torch.gather(tc, 1, b_sorted)
        step = max(int(info.get("t", 1)), 1)
        r = (r // step) * step
        assign, _ = self._select(r, a, b, a_sorted, b_sorted)
        nb = xb.shape[1]
        ridx = info["assign_b_indices"].clamp(0, nb - 1)
        rvalid = info["assign_valid_mask"]
        xb_contrib, wb_contrib = sparse_weighted_transport_pair(
            assign, (wa[..., None] * xa).contiguous(), wa.contiguous(), ridx, rvalid, nb)
        xb = wb[..., None] * xb + xb_contrib
        wb = wb + wb_contrib
        tmp = 1 - assign.sum(dim=-1)
        wa = wa * (tmp + (torch.clamp(tmp, 0.0, 1.0) - tmp).detach())
        wb_safe = torch.clamp(wb, min=torch.finfo(wb.dtype).eps)
        xb = xb / wb_safe[..., None]
        if trace_center:
            with torch.no_grad():
                c_contrib = sparse_weighted_transport(assign, (wa0 * ca.float()).unsqueeze(-1).contiguous(), ridx,
                                                      rvalid, nb)[..., 0]
                cb_new = (wb0 * cb.float() + c_contrib) / wb_safe
        x_out = torch.empty_like(x)
        size_out = torch.empty_like(size)
        if offset:
            x_out[:, :offset] = x[:, :offset]
            size_out[:, :offset] = size[:, :offset]
        if strided:
            x_out[:, ds] = xa.to(x.dtype)
            x_out[:, rs] = xb.to(x.dtype)
            size_out[:, ds, 0] = wa.to(size.dtype)
            size_out[:, rs, 0] = wb.to(size.dtype)
        else:
            x_out[:, offset:n] = x[:, offset:n]
            x_out.scatter_(1, a_sorted.unsqueeze(-1).expand(-1, -1, c), xa.to(x.dtype))
            x_out.scatter_(1, b_sorted.unsqueeze(-1).expand(-1, -1, c), xb.to(x.dtype))
            size_out[:, offset:n] = size[:, offset:n]
            size_out[..., 0].scatter_(1, a_sorted, wa.to(size.dtype))
            size_out[..., 0].scatter_(1, b_sorted, wb.to(size.dtype))
        if n < t_tokens:
            x_out[:, n:] = x[:, n:]
            size_out[:, n:] = size[:, n:]
        if trace_center:
            self._store_center(info, tc, ca, cb_new, a_sorted, b_sorted, ds if strided else None,
                               rs if strided else None, offset, n, bsz, t_tokens, dev)
        return x_out, size_out, n, None, None  # _select's out dict is None on the soft-k-max path

    @torch.no_grad()
    def _store_center(self, info, tc, ca, cb_new, a_sorted, b_sorted, ds, rs, offset, n, bsz, t_tokens, dev):
        """token_center after the layer (dtem.py:2031-2044 and the restore)."""
        old = info.get("token_center")
        center = torch.empty(bsz, t_tokens, device=dev, dtype=torch.float32)
        if offset:
            center[:, :offset] = 0 if old is None else old[:, :offset]
        if n < t_tokens:
            center[:, n:] = tc[:, n:]
        if ds is not None:
            center[:, ds] = ca.float()
            center[:, rs] = cb_new
        else:
            center.scatter_(1, a_sorted, ca.float())
            center.scatter_(1, b_sorted, cb_new)
        info["token_center"] = center


def make_merge_block(grid_size, radius=3.0, device=None, eval_grouping="alternating_per_layer_fast", **kwargs):
    """A DTEMMergeBlock in eval mode with LocalEncoder-style ``_tome_info``
    for a patch grid (CLS first)."""
    block = DTEMMergeBlock(default_tome_info(grid_size, radius, device=device, eval_grouping=eval_grouping, **kwargs))
    return block.eval()


__all__ = ["DTEMMergeBlock", "build_eval_group_indices", "default_tome_info", "make_merge_block",
           "build_patch_spatial_adjacency"]
