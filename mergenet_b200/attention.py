"""Windowed local attention on the B200 kernels, behind the reference's
function signatures (opentome/timm/bias_local_attn.py:243-625)."""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib as L


_STATUS = {}


def _status(dev):
    """Per-device status word the attention kernels OR error bits into."""
    key = (dev.type, dev.index)
    if key not in _STATUS:
        _STATUS[key] = torch.zeros(1, dtype=torch.int32, device=dev)
    return _STATUS[key]


def attention_status(device=None, reset=False):
    """Error bits recorded by attention kernels on ``device`` (sticky until
    reset; reading synchronises)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = _status(dev)
    val = int(st.item())
    if reset:
        st.zero_()
    return val


def _strides_bnhd(t: torch.Tensor):
    if t.stride(-1) != 1:
        raise ValueError("the head dimension must be contiguous")
    return t.stride(0), t.stride(1), t.stride(2)


HEAD_DIM = 64  # the tensor-core kernels' head width (the canonical 384 / 6 heads)


def _check_head_dim(d):
    if d != HEAD_DIM:
        raise ValueError(f"head_dim {d} is not supported: the B200 attention kernels take head_dim {HEAD_DIM} "
                         "(fp16 / bf16 on the tensor cores)")


def _tc_ready(t):
    """fp16 / bf16 with 16-byte aligned rows (what the TMA tensor maps need)."""
    return (t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0)


def _launch(q, k, v, bias, window, cls_global, scale, out_dtype):
    """q/k/v in (B, N, H, D) view form (any strides with a unit last stride)."""
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"q/k/v shape mismatch: {q.shape}, {k.shape}, {v.shape}")
    if bias is not None and tuple(bias.shape) != (q.shape[0], q.shape[1]):
        # the kernels read bias[b * N + j] for every key j of every image b
        raise ValueError(f"bias must be (B, N) = {(q.shape[0], q.shape[1])}, got {tuple(bias.shape)}")
    _check_head_dim(q.shape[-1])
    dev = L.require_cuda(q, k, v, bias)
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q/k/v must share a dtype")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"q/k/v must be float16 or bfloat16 for the tensor-core kernels, got {q.dtype}")
    if not (q.stride() == k.stride() == v.stride()):
        k = k.contiguous() if k.stride() != q.stride() else k
        v = v.contiguous() if v.stride() != q.stride() else v
        if not (q.stride() == k.stride() == v.stride()):
            q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if not (_tc_ready(q) and _tc_ready(k) and _tc_ready(v)):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    b, n, h, d = q.shape
    sb, sn, sh = _strides_bnhd(q)
    out = torch.empty(b, n, h, d, device=dev, dtype=out_dtype)
    bias_c = None
    bias_code = 0
    if bias is not None:
        bias_c = bias.contiguous()
        bias_code = L.dtype_code(bias_c.dtype)
    L.check(L.lib().mn_local_attention(b, n, h, d, L.dtype_code(q.dtype), L.ptr(q), L.ptr(k), L.ptr(v), sb, sn, sh,
                                       L.ptr(bias_c), bias_code, int(window), int(bool(cls_global)), float(scale),
                                       L.ptr(out), L.dtype_code(out_dtype), L.ptr(_status(dev)), L.stream_of(q)),
            "mn_local_attention")
    return out


def unbiased_local_attention(q, k, v, local_window, *, logical_dim: Optional[int] = None, dropout_p=0.0,
                             training=False, x_dtype: Optional[torch.dtype] = None, cls_global=False):
    """softmax(q k^T / sqrt(D)) v over keys with |i - j| <= local_window
    (bias_local_attn.py:486-625).  Layout inferred like the reference
    (BNHD when dim 1 > dim 2).  ``cls_global`` additionally makes row 0
    attend to every key (LocalAttention.forward, :704-719)."""
    if q.ndim != 4:
        raise AssertionError(f"q must be 4D, got shape {q.shape}")
    if training and dropout_p > 0.0:
        raise NotImplementedError("attention dropout is a training feature; the B200 path is inference")
    bnhd = q.shape[1] > q.shape[2]
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(logical_dim if logical_dim is not None else d)
    out_dtype = x_dtype if x_dtype is not None else q.dtype
    if q.dtype not in (torch.float16, torch.bfloat16):  # the reference casts to fp16 for its kernel (:533-537)
        q, k, v = q.half(), k.half(), v.half()
    if bnhd:
        return _launch(q, k, v, None, local_window, cls_global, scale, out_dtype)
    o = _launch(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None, local_window, cls_global, scale,
                out_dtype)
    return o.transpose(1, 2).contiguous()


def biased_local_attention(q, k, v, bias, local_window, *, logical_dim: Optional[int] = None, dropout_p=0.0,
                           training=False, x_dtype: Optional[torch.dtype] = None, input_layout: Optional[str] = None):
    """softmax(q k^T / sqrt(D) + bias_j) v over the window
    (bias_local_attn.py:243-483).  The bias is rounded to the q/k/v dtype as
    the reference's extra head column does.  Layout inference and its
    ambiguity error follow :321-347."""
    if q.ndim != 4:
        raise AssertionError(f"q must be 4D, got shape {q.shape}")
    if not (q.shape == k.shape == v.shape):
        raise AssertionError(f"q/k/v shape mismatch: {q.shape}, {k.shape}, {v.shape}")
    if not (bias.ndim == 2 and bias.shape[0] == q.shape[0]):
        raise AssertionError(f"bias must be 2D with matching batch size, got {bias.shape} for q={q.shape}")
    if input_layout is not None:
        input_layout = input_layout.upper()
        if input_layout not in ("BHND", "BNHD"):
            raise ValueError(f"input_layout must be BHND or BNHD, got {input_layout!r}")
    else:
        axis1_is_n = q.shape[1] == bias.shape[1]
        axis2_is_n = q.shape[2] == bias.shape[1]
        if axis1_is_n == axis2_is_n:
            raise ValueError("Cannot infer q/k/v layout from bias length; pass input_layout='BHND' or 'BNHD' "
                             "explicitly")
        input_layout = "BNHD" if axis1_is_n else "BHND"
    if training and dropout_p > 0.0:
        raise NotImplementedError("attention dropout is a training feature; the B200 path is inference")
    d_logic = logical_dim if logical_dim is not None else q.shape[-1]
    if d_logic < q.shape[-1] and q.shape[-1] % 8 != 0:
        # the reference's generic path (:416-483) then returns all D columns,
        # the ones past the logical width attention-weighted from v's padding
        raise ValueError(f"logical_dim {d_logic} below head_dim {q.shape[-1]} needs head_dim % 8 == 0 "
                         "(the reference's in-place bias-column layout)")
    scale = 1.0 / math.sqrt(d_logic)
    out_dtype = x_dtype if x_dtype is not None else q.dtype
    if q.dtype not in (torch.float16, torch.bfloat16):  # the reference computes in fp16 then
        q, k, v = q.half(), k.half(), v.half()
    if d_logic < q.shape[-1]:
        # columns past the logical width carry the bias / padding in the
        # reference's layout (:378-415); only the logical columns take part
        q, k, v = q[..., :d_logic], k[..., :d_logic], v[..., :d_logic]
    if input_layout == "BNHD":
        b, n = q.shape[0], q.shape[1]
        if bias.shape != (b, n):
            raise AssertionError(f"bias must be (B, N), got {bias.shape}")
        return _launch(q, k, v, bias, local_window, False, scale, out_dtype)
    b, n = q.shape[0], q.shape[2]
    if bias.shape != (b, n):
        raise AssertionError(f"bias must be (B, N), got {bias.shape}")
    o = _launch(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), bias, local_window, False, scale, out_dtype)
    return o.transpose(1, 2).contiguous()


def local_attention_packed(qkv, num_heads, local_window, cls_global=True, out_dtype=None, bias=None):
    """LocalAttention's core on the packed qkv projection [B, N, 3*H*D]
    (bias_local_attn.py:687-721 inference layout): q, k, v are read in place
    through strides; returns [B, N, H*D].  ``local_window < 0`` attends to
    every key; ``bias`` [B, N] adds a per-key bias (rounded to the qkv dtype,
    as SDPA's autocast rounds the float mask)."""
    b, n, c3 = qkv.shape
    if num_heads <= 0 or c3 % (3 * num_heads) != 0:
        raise ValueError(f"packed qkv width {c3} is not 3 x num_heads ({num_heads}) x head_dim")
    d = c3 // (3 * num_heads)
    view = qkv.view(b, n, 3, num_heads, d)
    q, k, v = view[:, :, 0], view[:, :, 1], view[:, :, 2]
    o = _launch(q, k, v, bias, local_window, cls_global, 1.0 / math.sqrt(d), out_dtype or qkv.dtype)
    return o.view(b, n, num_heads * d)


def cross_attention(q, k, v, scale=None, out_dtype=None, window=-1):
    """softmax(q k^T * scale) v with q [B, Nq, H, D] and k/v [B, Nk, H, D]
    (any strides with a unit last stride): the SDPA core of the recovery
    cross-attention (opentome/models/mergenet/model.py:173-188).  fp16 /
    bf16, head_dim 64 (the tensor-core kernel's contract)."""
    if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")
    _check_head_dim(q.shape[-1])
    dev = L.require_cuda(q, k, v)
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q/k/v must share a dtype")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"q/k/v must be float16 or bfloat16 for the tensor-core kernel, got {q.dtype}")
    if k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    if not _tc_ready(q):
        q = q.contiguous()
    if not (_tc_ready(k) and _tc_ready(v)):
        k, v = k.contiguous(), v.contiguous()
    b, nq, h, d = q.shape
    nk = k.shape[1]
    qsb, qsn, qsh = _strides_bnhd(q)
    ksb, ksn, ksh = _strides_bnhd(k)
    out_dtype = out_dtype or q.dtype
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    out = torch.empty(b, nq, h, d, device=dev, dtype=out_dtype)
    L.check(L.lib().mn_attention(b, nq, nk, h, d, L.dtype_code(q.dtype), L.ptr(q), qsb, qsn, qsh, L.ptr(k), L.ptr(v),
                                 ksb, ksn, ksh, int(window), scale, L.ptr(out), L.dtype_code(out_dtype),
                                 L.ptr(_status(dev)), L.stream_of(q)), "mn_attention")
    return out


class LocalAttention(torch.nn.Module):
    """Drop-in for the reference's LocalAttention module
    (opentome/timm/bias_local_attn.py:633-724): the same constructor
    arguments and parameter names (``qkv``, ``q_norm``, ``k_norm``, ``proj``),
    so its state dict loads as is.  The forward computes the qkv projection,
    then the windowed attention over the flat sequence with the global CLS
    row (``cls_global``) in one tensor-core kernel reading q/k/v in place from
    the packed projection, then the output projection.  As in the reference,
    fp32 q/k/v are rounded to fp16 for the attention (the reference's
    FlashAttention call); its CLS row is computed in the same kernel here.
    Inference only (attention dropout is a training feature)."""

    def __init__(self, dim, num_heads=8, qkv_bias=False, qk_norm=False, attn_drop=0.0, proj_drop=0.0,
                 norm_layer=torch.nn.LayerNorm, local_window=16, cls_global=False):
        super().__init__()
        if dim % num_heads != 0:
            raise AssertionError("dim should be divisible by num_heads")
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.fused_attn = False
        self.local_window = local_window
        self.cls_global = cls_global
        self.qkv = torch.nn.Linear(dim, dim * 3, bias=qkv_bias)
        self.q_norm = norm_layer(self.head_dim) if qk_norm else torch.nn.Identity()
        self.k_norm = norm_layer(self.head_dim) if qk_norm else torch.nn.Identity()
        self.attn_drop = torch.nn.Dropout(attn_drop)
        self.proj = torch.nn.Linear(dim, dim)
        self.proj_drop = torch.nn.Dropout(proj_drop)

    def forward(self, x):
        if self.training and self.attn_drop.p > 0.0:
            raise NotImplementedError("attention dropout is a training feature; the B200 path is inference")
        b, n, c = x.shape
        qkv = self.qkv(x)
        cls = self.cls_global and self.local_window >= 0 and n > 1
        if isinstance(self.q_norm, torch.nn.Identity) and isinstance(self.k_norm, torch.nn.Identity):
            packed = qkv if qkv.dtype in (torch.float16, torch.bfloat16) else qkv.half()
            out = local_attention_packed(packed, self.num_heads, self.local_window, cls_global=cls,
                                         out_dtype=qkv.dtype)
        else:
            q, k, v = qkv.view(b, n, 3, self.num_heads, self.head_dim).unbind(2)
            q, k = self.q_norm(q), self.k_norm(k)
            out = unbiased_local_attention(q, k, v, self.local_window, x_dtype=qkv.dtype,
                                           cls_global=cls).reshape(b, n, c)
        return self.proj_drop(self.proj(out))
