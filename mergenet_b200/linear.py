"""fp16 linear layers on the library's tcgen05 GEMM (``mn_gemm_f16``).

The block MLP and projections of mergenet_small_cls run under fp16 autocast
in the reference: ``F.linear`` on fp16 operands with an fp16 result, and
``nn.GELU`` (exact erf form) on that fp16 tensor (timm ``Mlp.forward``, as
the LocalBlock and latent blocks use it, opentome/timm/bias_local_attn.py:
859-869).  ``linear_f16`` computes the same values with fp32 accumulation in
tensor memory; ``gelu=True`` fuses the activation into the GEMM epilogue.
"""
from __future__ import annotations

import math

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


# ----------------------------------------------------------------------------
# fp32 linear layers as split-precision tcgen05 GEMMs (mn_gemm_f32_split)
# ----------------------------------------------------------------------------
ACT_SCALE = 256.0  # activations are split after this exact power-of-two scaling


class SplitWeight:
    """An nn.Linear weight [N, K] (and fp32 bias) held as the fp16 pair the
    split-precision GEMM takes: w * 2^e = hi + lo, with 2^e chosen so the
    largest entry is near 2^10 (both halves stay in fp16's normal range for
    all but the smallest weights, whose lo parts are below 2^-24 of the
    scaled maximum)."""

    def __init__(self, weight, bias=None):
        w = weight.detach().float()
        amax = float(w.abs().max()) if w.numel() else 0.0
        self.exp = int(math.floor(math.log2(1024.0 / amax))) if amax > 0 else 0
        ws = w * (2.0 ** self.exp)
        self.hi = ws.half().contiguous()
        self.lo = (ws - self.hi.float()).half().contiguous()
        self.bias = None if bias is None else bias.detach().float().contiguous()
        self.out_features, self.in_features = w.shape


def layernorm_split(x, ln, scale=ACT_SCALE):
    """(hi, lo) fp16 planes of LayerNorm(x) * scale for fp32 x [..., C]."""
    L.require_cuda(x)
    if x.dtype != torch.float32:
        raise TypeError("layernorm_split takes float32 x")
    c = x.shape[-1]
    x2 = x.reshape(-1, c).contiguous()
    hi = torch.empty(x2.shape, device=x.device, dtype=torch.float16)
    lo = torch.empty_like(hi)
    L.check(L.lib().mn_layernorm_split(x2.shape[0], c, L.ptr(x2), L.ptr(ln.weight), L.ptr(ln.bias), float(ln.eps),
                                       float(scale), L.ptr(hi), L.ptr(lo), L.stream_of(x)), "mn_layernorm_split")
    return hi.view(x.shape), lo.view(x.shape)


def linear_f32_split(a_hi, a_lo, weight: SplitWeight, a_scale=ACT_SCALE, out_dtype=torch.float32, out=None):
    """y = (A / a_scale) @ W^T + bias in fp32-equivalent precision, with A
    given as fp16 planes a_hi (+ a_lo, or None when A is exactly fp16):
    three tcgen05 MMAs per K step into one fp32 accumulator.  Returns
    [..., N] in out_dtype (float32 or float16)."""
    L.require_cuda(a_hi, a_lo)
    k = a_hi.shape[-1]
    if k != weight.in_features:
        raise ValueError(f"weight has {weight.in_features} inputs, A has {k}")
    a2 = a_hi.reshape(-1, k)
    l2 = None if a_lo is None else a_lo.reshape(-1, k)
    if a2.stride(1) != 1 or (l2 is not None and (l2.stride(1) != 1 or l2.stride(0) != a2.stride(0))):
        a2 = a2.contiguous()
        l2 = None if l2 is None else l2.contiguous()
    n = weight.out_features
    if out is None:
        out = torch.empty(*a_hi.shape[:-1], n, device=a_hi.device, dtype=out_dtype)
    o2 = out.view(-1, n)
    dev = a_hi.device
    for t in (weight.hi, weight.lo, weight.bias):
        if t is not None and t.device != dev:
            raise ValueError("split weight and activations must be on the same device")
    scale = 1.0 / (float(a_scale) * (2.0 ** weight.exp))
    L.check(L.lib().mn_gemm_f32_split(a2.shape[0], n, k, L.ptr(a2), L.ptr(l2), a2.stride(0), L.ptr(weight.hi),
                                      L.ptr(weight.lo), weight.hi.stride(0), L.ptr(weight.bias), scale, L.ptr(o2),
                                      o2.stride(0), L.dtype_code(out.dtype), L.ptr(_status(dev)),
                                      L.stream_of(a_hi)), "mn_gemm_f32_split")
    return out
