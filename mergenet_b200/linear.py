"""fp16 linear layers on the library's tcgen05 GEMM (``mn_gemm_f16``).

The block MLP and projections of mergenet_small_cls run under fp16 autocast
in the reference: ``F.linear`` on fp16 operands with an fp16 result, and
``nn.GELU`` (exact erf form) on that fp16 tensor (timm ``Mlp.forward``, as
the LocalBlock and latent blocks use it, opentome/timm/bias_local_attn.py:
859-869).  ``linear_f16`` computes the same values with fp32 accumulation in
tensor memory; ``gelu=True`` fuses the activation into the GEMM epilogue.
"""
from __future__ import annotations

import torch

from . import _lib as L


def linear_f16(x, weight, bias=None, gelu=False, out=None):
    """y = x @ weight^T + bias (then GELU) for fp16 CUDA tensors.

    x [..., K] (rows contiguous), weight [N, K], bias [N] or None; returns
    [..., N] fp16 (written into ``out`` when given).  K must be a multiple of
    64 and N of 128."""
    L.require_cuda(x, weight, bias)
    if x.dtype != torch.float16 or weight.dtype != torch.float16 or (bias is not None and bias.dtype != torch.float16):
        raise TypeError("linear_f16 takes float16 x, weight and bias")
    k = x.shape[-1]
    n = weight.shape[0]
    if weight.shape[1] != k:
        raise ValueError(f"weight {tuple(weight.shape)} does not match x [..., {k}]")
    if bias is not None and bias.shape != (n,):
        raise ValueError(f"bias {tuple(bias.shape)} does not match N = {n}")
    x2 = x.reshape(-1, k)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    w = weight if weight.stride(1) == 1 else weight.contiguous()
    b = None if bias is None else bias.contiguous()
    m = x2.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], n, device=x.device, dtype=torch.float16)
    o2 = out.view(-1, n)
    status = _status(x.device)
    L.check(L.lib().mn_gemm_f16(m, n, k, L.ptr(x2), x2.stride(0), L.ptr(w), w.stride(0), L.ptr(b),
                                L.MN_EPI_BIAS_GELU if gelu else L.MN_EPI_BIAS, L.ptr(o2), o2.stride(0),
                                L.ptr(status), L.stream_of(x)), "mn_gemm_f16")
    return out


_STATUS = {}


def _status(dev):
    key = (dev.type, dev.index)
    if key not in _STATUS:
        _STATUS[key] = torch.zeros(1, dtype=torch.int32, device=dev)
    return _STATUS[key]


def gemm_status(device=None, reset=False):
    """Error bits recorded by the GEMM on ``device`` (sticky until reset)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = _status(dev)
    val = int(st.item())
    if reset:
        st.zero_()
    return val
