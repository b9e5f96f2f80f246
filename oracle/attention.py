"""numpy restatement of the reference's windowed attention (the oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Follows the naive unfold implementations naive_unbiased_local_attention /
naive_biased_local_attention (opentome/timm/bias_local_attn.py:46-240): key j
takes part in query i's softmax iff |i - j| <= window, the per-key bias is
added to q.k / sqrt(D), computed here in float64.  ``cls_global`` adds the
CLS row of LocalAttention.forward (:704-719): row 0 attends to every key.
"""
from __future__ import annotations

import numpy as np


def local_attention(q, k, v, window, bias=None, cls_global=False, scale=None):
    """q, k, v [B, N, H, D] (BNHD); bias [B, N] or None -> out [B, N, H, D] f64."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    b, n, h, d = q.shape
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    s = np.einsum("bihd,bjhd->bhij", q, k) * scale
    if bias is not None:
        s = s + np.asarray(bias, np.float64)[:, None, None, :]
    pos = np.arange(n)
    allowed = np.abs(pos[:, None] - pos[None, :]) <= window if window >= 0 else np.ones((n, n), bool)
    allowed = np.broadcast_to(allowed, s.shape).copy()
    if cls_global and window >= 0 and n > 1:
        allowed[:, :, 0, :] = True
    s = np.where(allowed, s, -np.inf)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    return np.einsum("bhij,bjhd->bihd", p, v)
