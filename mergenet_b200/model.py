"""mergenet_small_cls inference on the B200 kernels.

Module tree and parameter names follow the reference's
CLSHybridToMeModel built by ``mergenet_small_cls`` (opentome/models/mergenet/
model.py:1602-1607 with the canonical kwargs :24-53): ``local.vit.*`` (patch
embed, CLS, position embedding, six LocalBlocks), ``local.metric_layers.*``,
``encode_cross_attention.*``, ``latent.vit.*`` (six global blocks + norm) and
``head``, so a reference state dict maps onto it key for key.

The forward is the reference's inference path under fp16 autocast
(model.py:1141-1222): fp16 GEMMs and attention inside fp32 residual
streams, fp32 LayerNorm statistics, fp32 routing.  The hot path runs on the
library: windowed local attention with the CLS row (bias_local_attn.py:
679-724), the fused six-layer routing + carrier gather (model.py:574-590,
:1157-1183), the cross-attention core (model.py:173-188), the latent blocks'
proportional attention (opentome/timm/tome.py:44-58) and the fused residual
add + LayerNorm + fp16 cast around every block.  GEMMs and GELU are cuBLAS /
ATen.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import cross_attention, local_attention_packed
from .routing import RoutePlan


class _PatchEmbed(nn.Module):
    def __init__(self, patch, dim):
        super().__init__()
        self.proj = nn.Conv2d(3, dim, patch, patch)


class _Attention(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.qkv = nn.Linear(dim, dim * 3)
        self.proj = nn.Linear(dim, dim)


class _Mlp(nn.Module):
    def __init__(self, dim, hidden):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.fc2 = nn.Linear(hidden, dim)


class _Block(nn.Module):
    def __init__(self, dim, mlp_ratio, eps=1e-5):
        super().__init__()
        self.norm1 = nn.LayerNorm(dim, eps=eps)
        self.attn = _Attention(dim)
        self.norm2 = nn.LayerNorm(dim, eps=eps)
        self.mlp = _Mlp(dim, int(dim * mlp_ratio))


class _LocalVit(nn.Module):
    def __init__(self, img, patch, dim, depth, mlp_ratio):
        super().__init__()
        self.patch_embed = _PatchEmbed(patch, dim)
        n = (img // patch) ** 2
        self.cls_token = nn.Parameter(torch.zeros(1, 1, dim))
        self.pos_embed = nn.Parameter(torch.zeros(1, n + 1, dim))
        self.blocks = nn.ModuleList([_Block(dim, mlp_ratio) for _ in range(depth)])


class _Local(nn.Module):
    def __init__(self, img, patch, dim, depth, mlp_ratio, metric_dim):
        super().__init__()
        self.vit = _LocalVit(img, patch, dim, depth, mlp_ratio)
        self.metric_layers = nn.ModuleList([nn.Linear(dim, metric_dim) for _ in range(depth)])


class _LatentVit(nn.Module):
    def __init__(self, img, patch, dim, depth, mlp_ratio):
        super().__init__()
        self.pos_embed = nn.Parameter(torch.zeros(1, (img // patch) ** 2, dim), requires_grad=False)
        # timm VisionTransformer blocks and final norm use LayerNorm(eps=1e-6)
        self.blocks = nn.ModuleList([_Block(dim, mlp_ratio, eps=1e-6) for _ in range(depth)])
        self.norm = nn.LayerNorm(dim, eps=1e-6)


class _Latent(nn.Module):
    def __init__(self, img, patch, dim, depth, mlp_ratio):
        super().__init__()
        self.vit = _LatentVit(img, patch, dim, depth, mlp_ratio)


class CrossAttention(nn.Module):
    """MyCrossAttention (model.py:90-221) parameters."""

    def __init__(self, dim, heads):
        super().__init__()
        self.num_heads = heads
        self.q_norm = nn.LayerNorm(dim)
        self.kv_norm = nn.LayerNorm(dim)
        self.q_proj = nn.Linear(dim, dim)
        self.k_proj = nn.Linear(dim, dim)
        self.v_proj = nn.Linear(dim, dim)
        self.out_proj = nn.Linear(dim, dim)


class MergeNetSmall(nn.Module):
    """Canonical MN-L2-R3 classifier (dim 384, 6 heads, 6 local + 6 latent)."""

    def __init__(self, img_size=224, patch_size=8, embed_dim=384, num_heads=6, mlp_ratio=4.0, local_depth=6,
                 latent_depth=6, num_classes=1000, metric_dim=64, spatial_radius=3.0, local_window=16,
                 lambda_local=2.0):
        super().__init__()
        self.img_size, self.patch_size = img_size, patch_size
        self.embed_dim, self.num_heads = embed_dim, num_heads
        self.local_window = local_window
        self.spatial_radius = spatial_radius
        self.grid = (img_size // patch_size, img_size // patch_size)
        num_patches = self.grid[0] * self.grid[1]
        self.total_merge_local = int(num_patches * (lambda_local - 1) / lambda_local)
        default_r = self.total_merge_local // max(local_depth, 1)
        r_list = [default_r] * local_depth  # parse_r(local_depth, default_r, total) (tome.py:12-53)
        r_list[-1] += self.total_merge_local - sum(r_list)
        self.r_list = r_list
        self.local = _Local(img_size, patch_size, embed_dim, local_depth, mlp_ratio, metric_dim)
        self.latent = _Latent(img_size, patch_size, embed_dim, latent_depth, mlp_ratio)
        self.head = nn.Linear(embed_dim, num_classes)
        self.encode_cross_attention = CrossAttention(embed_dim, num_heads)
        self._plans = {}
        self._half = None
        self._kv16 = None
        self._patch_w16 = None

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def init_weights(self, seed=0):
        """Random init in the reference's style: timm ViT init for the ViT
        parts (trunc-normal 0.02 linears, zero biases, CLS ~ N(0, 1e-6)),
        PyTorch defaults for the metric heads and cross-attention, zero
        cross-attention output projection (model.py:822-829)."""
        g = torch.Generator().manual_seed(seed)

        def tn(t, std=0.02):
            t.copy_(torch.nn.init.trunc_normal_(torch.empty_like(t), std=std, generator=g))

        for vit in (self.local.vit, self.latent.vit):
            tn(vit.pos_embed)
            for blk in vit.blocks:
                for lin in (blk.attn.qkv, blk.attn.proj, blk.mlp.fc1, blk.mlp.fc2):
                    tn(lin.weight)
                    lin.bias.zero_()
        self.local.vit.cls_token.normal_(0, 1e-6, generator=g)
        pe = self.local.vit.patch_embed.proj
        bound = 1 / math.sqrt(pe.weight[0].numel())
        pe.weight.uniform_(-bound, bound, generator=g)
        pe.bias.uniform_(-bound, bound, generator=g)
        for lin in list(self.local.metric_layers) + [self.encode_cross_attention.q_proj,
                                                      self.encode_cross_attention.k_proj,
                                                      self.encode_cross_attention.v_proj]:
            bound = 1 / math.sqrt(lin.in_features)
            lin.weight.uniform_(-bound, bound, generator=g)
            lin.bias.uniform_(-bound, bound, generator=g)
        self.encode_cross_attention.out_proj.weight.zero_()
        self.encode_cross_attention.out_proj.bias.zero_()
        tn(self.head.weight)
        self.head.bias.zero_()
        self._half = None
        self._kv16 = None
        self._patch_w16 = None
        return self

    # ------------------------------------------------------------- execution
    def _plan(self, device):
        key = (device.type, device.index)
        if key not in self._plans:
            self._plans[key] = RoutePlan(self.grid, self.spatial_radius, self.r_list, device=device)
        return self._plans[key]

    def _weights16(self):
        """fp16 copies of the GEMM weights autocast would cast on every call."""
        if self._half is None:
            self._half = {n: p.detach().half() for n, p in self.named_parameters()
                          if p.ndim >= 2 and "pos_embed" not in n and "cls_token" not in n}
        return self._half

    def _linear16(self, x, name, lin):
        w = self._weights16()[name + ".weight"]
        return F.linear(x.half(), w, lin.bias.half())

    def _metric(self, h_raw, i, metrics, w16):
        lin = self.local.metric_layers[i]
        torch.addmm(lin.bias.half(), h_raw.view(-1, h_raw.shape[-1]), w16[f"local.metric_layers.{i}.weight"].t(),
                    out=metrics[i].view(-1, metrics.shape[-1]))

    def _attn_local(self, h, i, blk):
        qkv = self._linear16(h, f"local.vit.blocks.{i}.attn.qkv", blk.attn.qkv)
        a = local_attention_packed(qkv, self.num_heads, self.local_window, cls_global=True)
        return self._linear16(a, f"local.vit.blocks.{i}.attn.proj", blk.attn.proj)

    def _attn_latent(self, h, i, blk, log_size):
        # ToMeAttention with proportional attention (opentome/timm/tome.py:44-58):
        # softmax(q k^T / sqrt(d) + log size_j) v over all carriers
        qkv = self._linear16(h, f"latent.vit.blocks.{i}.attn.qkv", blk.attn.qkv)
        a = local_attention_packed(qkv, self.num_heads, -1, cls_global=False, bias=log_size)
        return self._linear16(a, f"latent.vit.blocks.{i}.attn.proj", blk.attn.proj)

    def _mlp(self, h, prefix, blk):
        # fc1 + GELU in one cuBLASLt call (bias + GELU epilogue; its GELU agrees
        # with the exact erf GELU to within fp16 output rounding)
        w16 = self._weights16()
        shp = h.shape
        f = torch._addmm_activation(blk.mlp.fc1.bias.half(), h.reshape(-1, shp[-1]),
                                    w16[prefix + ".mlp.fc1.weight"].t(), use_gelu=True)
        return self._linear16(f, prefix + ".mlp.fc2", blk.mlp.fc2).view(*shp[:-1], -1)

    def _cross(self, topk_x, x_embed):
        """MyCrossAttention (model.py:122-221).  The q/k/v projections feed an
        fp16 attention (SDPA autocasts its inputs), so they run as fp16 GEMMs
        with fp32 accumulation on LayerNorm outputs rounded to fp16; the
        out-projection keeps an fp32 result (TF32 tensor cores)."""
        ca = self.encode_cross_attention
        b, nq, c = topk_x.shape
        nk = x_embed.shape[1]
        hd = c // self.num_heads
        w16 = self._weights16()
        qn = add_layernorm(topk_x, None, ca.q_norm)[1]
        kvn = add_layernorm(x_embed, None, ca.kv_norm)[1]
        q = F.linear(qn, w16["encode_cross_attention.q_proj.weight"], ca.q_proj.bias.half())
        if self._kv16 is None:
            self._kv16 = (torch.cat([ca.k_proj.weight, ca.v_proj.weight]).half(),
                          torch.cat([ca.k_proj.bias, ca.v_proj.bias]).half())
        kv = F.linear(kvn, *self._kv16).view(b, nk, 2, self.num_heads, hd)
        ctx = cross_attention(q.view(b, nq, self.num_heads, hd), kv[:, :, 0], kv[:, :, 1], out_dtype=torch.float32)
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = True
        try:
            out = F.linear(ctx.view(b, nq, c), ca.out_proj.weight, ca.out_proj.bias)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        return out

    def _embed(self, images, w16):
        """timm PatchEmbed + _pos_embed: the non-overlapping patch conv as one
        GEMM over fp16 patch rows, written with the position embedding into
        the fp32 residual stream (CLS row first)."""
        vit = self.local.vit
        b, ch, hh, ww = images.shape
        p = self.patch_size
        gh, gw = hh // p, ww // p
        patches = torch.empty(b, gh, gw, ch, p, p, device=images.device, dtype=torch.float16)
        patches.copy_(images.view(b, ch, gh, p, gw, p).permute(0, 2, 4, 1, 3, 5))  # cast + unfold, one pass
        wpe = self._patch_w16
        if wpe is None:
            wpe = w16["local.vit.patch_embed.proj.weight"].reshape(self.embed_dim, -1).t().contiguous()
            self._patch_w16 = wpe
        emb = torch.addmm(vit.patch_embed.proj.bias.half(), patches.view(b * gh * gw, -1), wpe)
        x = torch.empty(b, gh * gw + 1, self.embed_dim, device=images.device, dtype=torch.float32)
        torch.add(emb.view(b, gh * gw, -1), vit.pos_embed[:, 1:], out=x[:, 1:])
        x[:, 0] = vit.cls_token[:, 0] + vit.pos_embed[:, 0]
        return x

    @torch.no_grad()
    def forward(self, images, return_intermediates=False):
        """images [B, 3, H, W] -> (logits [B, classes] fp16, aux dict).
        ``return_intermediates`` adds the tensors handed between stages
        (x_embed, metrics, topk_x, topk_size) to aux, for checking."""
        if not images.is_cuda:
            raise RuntimeError("MergeNetSmall runs on CUDA (there is no CPU path)")
        w16 = self._weights16()
        vit = self.local.vit
        b = images.shape[0]
        x = self._embed(images, w16)
        n, c = x.shape[1], x.shape[2]
        depth = len(vit.blocks)
        metrics = torch.empty(depth, b, n, self.local.metric_layers[0].out_features, device=x.device,
                              dtype=torch.float16)
        y = None
        for i, blk in enumerate(vit.blocks):
            # x <- x + y (previous MLP), h = LN1(x); fp16(x) feeds the previous metric head
            _, h, raw = add_layernorm(x, y, blk.norm1, x_out=x if y is not None else None, want_raw=i > 0)
            if i > 0:
                self._metric(raw, i - 1, metrics, w16)
            p = self._attn_local(h, i, blk)
            _, h, _ = add_layernorm(x, p, blk.norm2, x_out=x)
            y = self._mlp(h, f"local.vit.blocks.{i}", blk)
        _, _, raw = add_layernorm(x, y, None, x_out=x, want_ln=False, want_raw=True)
        self._metric(raw, depth - 1, metrics, w16)
        x_embed = x
        route = self._plan(x.device)(x_embed, metrics)
        topk_x = route.topk_x
        x_trace = self._cross(topk_x, x_embed) + topk_x
        log_size = route.topk_size.log()
        y = None
        for i, blk in enumerate(self.latent.vit.blocks):
            _, h, _ = add_layernorm(x_trace, y, blk.norm1, x_out=x_trace if y is not None else None)
            p = self._attn_latent(h, i, blk, log_size)
            _, h, _ = add_layernorm(x_trace, p, blk.norm2, x_out=x_trace)
            y = self._mlp(h, f"latent.vit.blocks.{i}", blk)
        lv = self.latent.vit
        cls = x_trace[:, 0] + y[:, 0].float()
        cls = F.layer_norm(cls, (c,), lv.norm.weight, lv.norm.bias, lv.norm.eps)
        logits = self._linear16(cls, "head", self.head)
        aux = {
            "token_strength_no_cls": route.size[:, 1:],
            "topk_patch_indices": route.topk_idx,
            "retained_tokens": int(route.topk_idx.shape[1]),
            "cls_feature": cls,
        }
        if return_intermediates:
            aux.update(x_embed=x_embed, metrics=metrics, topk_x=topk_x, topk_size=route.topk_size,
                       token_center=route.center)
        return logits, aux


def add_layernorm(x, y, ln, x_out=None, want_ln=True, want_raw=False):
    """(x + y [fp32], LayerNorm(x + y) [fp16], fp16(x + y)) in one pass of the
    library's fused kernel; y (fp16) may be None, outputs not wanted are None."""
    from . import _lib as L
    c = x.shape[-1]
    rows = x.numel() // c
    h_ln = torch.empty(x.shape, device=x.device, dtype=torch.float16) if want_ln else None
    h_raw = torch.empty(x.shape, device=x.device, dtype=torch.float16) if want_raw else None
    if y is not None and y.dtype != torch.float16:
        y = y.half()
    L.check(L.lib().mn_add_layernorm(rows, c, L.ptr(x), L.ptr(y), L.ptr(ln.weight) if want_ln else None,
                                     L.ptr(ln.bias) if want_ln else None, float(ln.eps) if want_ln else 0.0,
                                     L.ptr(x_out), L.ptr(h_ln), L.ptr(h_raw), L.stream_of(x)), "mn_add_layernorm")
    return x_out, h_ln, h_raw


def mergenet_small_cls(**kwargs):
    """Factory with the reference's canonical single-branch defaults."""
    return MergeNetSmall(**kwargs)
