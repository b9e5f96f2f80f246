"""CPU stand-in for FlashAttention's ``flash_attn_func``, written for this
repository and used ONLY by tests/golden/make_model_golden.py, which runs the
reference model on the host.  FlashAttention is a CUDA library; this computes
what its documentation specifies for the arguments the reference passes --
softmax(q k^T * softmax_scale) v over keys with -w_left <= j - i <= w_right
(a negative side is unbounded) -- in fp32 on [B, N, H, D] tensors, returning
the input dtype.
"""
import math

import torch


def flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
                    deterministic=False, **_):
    if dropout_p:
        raise NotImplementedError("the stand-in has no dropout")
    b, n, h, d = q.shape
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(d)
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))  # [B, H, N, D]
    s = (qf @ kf.transpose(-1, -2)) * scale
    pos = torch.arange(n)
    rel = pos[None, :] - pos[:, None]  # j - i
    left, right = window_size
    allowed = torch.ones(n, n, dtype=torch.bool)
    if left >= 0:
        allowed &= rel >= -left
    if right >= 0:
        allowed &= rel <= right
    if causal:
        allowed &= rel <= 0
    s = s.masked_fill(~allowed, float("-inf"))
    out = torch.softmax(s, dim=-1) @ vf
    return out.transpose(1, 2).to(q.dtype)


flash_attn_interface = None
