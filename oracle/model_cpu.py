"""CPU port of the mergenet_small_cls inference forward (timed CPU baseline).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Used by ``bench.py``
for its CPU-baseline leg and ``--impl reference`` arm: the reference itself
cannot run on a host without its GPU-only FlashAttention and without timm, so
this port restates its forward (opentome/models/mergenet/model.py:1141-1222)
on the host cores in float32 with batched torch CPU ops: the dense layers,
the windowed attention of bias_local_attn.py:679-724 on the band only (plus
the global CLS row), the six merge layers and the carrier block as the
reference's sparse CPU path computes them (``route_torch``), SDPA-equivalent
cross- and latent attention.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import routing as R


def _band_attention(q, k, v, window, cls_global):
    """softmax(q k^T / sqrt(D)) v over keys |i - j| <= window, computed on the
    band only (the 2w + 1 keys of each query gathered with unfold), plus the
    global CLS row; q/k/v [B, H, N, D]."""
    b, h, n, d = q.shape
    w = int(window)
    scale = d ** -0.5
    kp = F.pad(k, (0, 0, w, w))
    vp = F.pad(v, (0, 0, w, w))
    kw = kp.unfold(2, 2 * w + 1, 1)  # [B, H, N, D, 2w+1]
    vw = vp.unfold(2, 2 * w + 1, 1)
    s = torch.einsum("bhnd,bhndw->bhnw", q, kw) * scale
    pos = torch.arange(n)[:, None] + torch.arange(-w, w + 1)[None, :]
    s = s.masked_fill(((pos < 0) | (pos >= n))[None, None], float("-inf"))
    out = torch.einsum("bhnw,bhndw->bhnd", torch.softmax(s, -1), vw)
    if cls_global and n > 1:
        out = out.clone()
        out[:, :, :1] = torch.softmax((q[:, :, :1] @ k.transpose(-1, -2)) * scale, -1) @ v
    return out


def _thre_topk(x, k, temperature=30.0):
    """ThreTopK (opentome/utils/thetopk.py:4-43) in torch: one global range,
    sorted rows, the two log-cum-sum-exp scans, the first bracket."""
    x = x / (x.max() - x.min()) * temperature
    n = x.shape[1]
    xs, _ = torch.sort(x, dim=-1)
    lse1 = torch.logcumsumexp(xs, dim=-1)
    lse2 = torch.logcumsumexp(-xs.flip(-1), dim=-1).flip(-1)
    lse2 = torch.cat([lse2[:, 1:], torch.full_like(lse2[:, :1], float("-inf"))], 1)
    k_m = (k - torch.arange(n - 1, -1, -1)).to(x.dtype)
    term = torch.sqrt(k_m * k_m + torch.exp(lse1 + lse2)) + k_m
    x_lamb = lse1 - torch.log(term.abs() + 1e-8)
    shift = torch.cat([xs[:, 1:], torch.full_like(xs[:, :1], float("inf"))], 1)
    idx = ((x_lamb >= xs) & (x_lamb <= shift)).to(torch.uint8).argmax(-1, keepdim=True)
    delta = x - x_lamb.gather(1, idx)
    return torch.where(delta > 0, 1 - 0.5 * torch.exp(-delta), 0.5 * torch.exp(delta))


def route_torch(x, metrics, r_list, geom, tau1=1.0, tau2=30.0):
    """The six soft-merge layers and the carrier block with batched torch ops
    on the host, the way the reference's sparse CPU path computes them
    (dtem.py:1687-2223 with the alternating_per_layer_fast grouping; scores
    from gathered receiver rows, the soft-k-max block, the transport as one
    scatter_add per layer; model.py:1157-1183 for the carriers).  For the
    timed baseline; the numpy oracle is the checker."""
    b, t, c = x.shape
    nbr = torch.from_numpy(geom.nbr_idx).long()
    nval = torch.from_numpy(geom.nbr_valid)
    size = torch.ones(b, t)
    center = torch.arange(t, dtype=torch.float32).expand(b, t).clone()
    x = x.clone()
    for layer, r in enumerate(r_list):
        m = metrics[layer].float()
        m = m / m.norm(dim=-1, keepdim=True).clamp_min(1e-6)
        dp = 0 if layer % 2 else 1  # donor patch parity
        rp = 1 - dp
        ds, rs = slice(1 + dp, t, 2), slice(1 + rp, t, 2)
        xa, xb, a, bm = x[:, ds].clone(), x[:, rs].clone(), m[:, ds], m[:, rs]
        wa, wb, ca, cb = size[:, ds].clone(), size[:, rs].clone(), center[:, ds].clone(), center[:, rs].clone()
        na, nb = xa.shape[1], xb.shape[1]
        dpatch = torch.arange(na) * 2 + dp
        rpatch = nbr[dpatch]  # [Na, K]
        allowed = nval[dpatch] & (rpatch % 2 == rp)
        ridx = torch.where(allowed, (rpatch - rp) // 2, torch.zeros_like(rpatch))
        scores = torch.einsum("bnc,bnkc->bnk", a, bm[:, ridx.reshape(-1)].view(b, na, -1, bm.shape[-1]))
        allowed = allowed.expand(b, -1, -1)
        valid_row = allowed.any(-1)
        logits = (scores / tau1).masked_fill(~allowed, float("-inf"))
        safe = torch.where(valid_row[..., None], logits, torch.zeros_like(logits))
        energy = torch.where(valid_row, torch.logsumexp(safe, -1).exp(), torch.zeros_like(valid_row, dtype=torch.float32))
        row_khot = _thre_topk(energy, int(min(r, (t - 1) // 2)), tau2) * valid_row
        khot = torch.softmax(safe, -1) * allowed * row_khot[..., None]
        assign = khot / ((khot.sum(-1, keepdim=True) - 1).clamp_min(0) + 1)
        idx = ridx.reshape(1, -1).expand(b, -1)
        contrib = (assign[..., None] * (wa[..., None] * xa)[:, :, None, :]).reshape(b, -1, c)
        xb_c = torch.zeros(b, nb, c).scatter_add_(1, idx[..., None].expand(-1, -1, c), contrib)
        wb_c = torch.zeros(b, nb).scatter_add_(1, idx, (assign * wa[..., None]).reshape(b, -1))
        cb_c = torch.zeros(b, nb).scatter_add_(1, idx, (assign * (wa * ca)[..., None]).reshape(b, -1))
        wb_new = wb + wb_c
        wb_safe = wb_new.clamp_min(torch.finfo(torch.float32).eps)
        x[:, rs] = (wb[..., None] * xb + xb_c) / wb_safe[..., None]
        size[:, ds] = wa * (1 - assign.sum(-1)).clamp(0, 1)
        size[:, rs] = wb_new
        center[:, rs] = (wb * cb + cb_c) / wb_safe
        center[:, 0] = 0
    k = t - 1 - sum(r_list)
    _, top = torch.topk(size[:, 1:], k, dim=1, sorted=False)
    order = torch.argsort(torch.gather(center[:, 1:], 1, top), dim=1)
    top = torch.gather(top, 1, order)
    topk_x = torch.cat([x[:, :1], torch.gather(x, 1, (top + 1)[..., None].expand(-1, -1, c))], 1)
    topk_size = torch.cat([size[:, :1], torch.gather(size, 1, top + 1)], 1)
    return topk_x, topk_size, top


def forward(model, images, geometry=None):
    """model: a mergenet_b200.model.MergeNetSmall (weights read on the CPU);
    images [B, 3, H, W] float32 CPU -> logits [B, classes] float32."""
    sd = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
    heads = model.num_heads
    b = images.shape[0]
    p = model.patch_size
    x = F.conv2d(images.float(), sd["local.vit.patch_embed.proj.weight"], sd["local.vit.patch_embed.proj.bias"],
                 stride=p)
    x = x.flatten(2).transpose(1, 2)
    x = torch.cat([sd["local.vit.cls_token"].expand(b, -1, -1), x], 1) + sd["local.vit.pos_embed"]
    n, c = x.shape[1], x.shape[2]
    hd = c // heads
    metrics = []
    depth = len(model.local.vit.blocks)
    for i in range(depth):
        pre = f"local.vit.blocks.{i}."
        h = F.layer_norm(x, (c,), sd[pre + "norm1.weight"], sd[pre + "norm1.bias"])
        qkv = F.linear(h, sd[pre + "attn.qkv.weight"], sd[pre + "attn.qkv.bias"])
        q, k, v = qkv.view(b, n, 3, heads, hd).permute(2, 0, 3, 1, 4).unbind(0)
        a = _band_attention(q, k, v, model.local_window, True).transpose(1, 2).reshape(b, n, c)
        x = x + F.linear(a, sd[pre + "attn.proj.weight"], sd[pre + "attn.proj.bias"])
        h = F.layer_norm(x, (c,), sd[pre + "norm2.weight"], sd[pre + "norm2.bias"])
        h = F.gelu(F.linear(h, sd[pre + "mlp.fc1.weight"], sd[pre + "mlp.fc1.bias"]))
        x = x + F.linear(h, sd[pre + "mlp.fc2.weight"], sd[pre + "mlp.fc2.bias"])
        metrics.append(F.linear(x, sd[f"local.metric_layers.{i}.weight"], sd[f"local.metric_layers.{i}.bias"]))
    geom = geometry or R.Geometry(model.grid, model.spatial_radius)
    topk_x, topk_size, topk_idx = route_torch(x, metrics, model.r_list, geom)
    pre = "encode_cross_attention."
    qn = F.layer_norm(topk_x, (c,), sd[pre + "q_norm.weight"], sd[pre + "q_norm.bias"])
    kvn = F.layer_norm(x, (c,), sd[pre + "kv_norm.weight"], sd[pre + "kv_norm.bias"])
    q = F.linear(qn, sd[pre + "q_proj.weight"], sd[pre + "q_proj.bias"]).view(b, -1, heads, hd).transpose(1, 2)
    k = F.linear(kvn, sd[pre + "k_proj.weight"], sd[pre + "k_proj.bias"]).view(b, n, heads, hd).transpose(1, 2)
    v = F.linear(kvn, sd[pre + "v_proj.weight"], sd[pre + "v_proj.bias"]).view(b, n, heads, hd).transpose(1, 2)
    ctx = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(b, -1, c)
    xt = F.linear(ctx, sd[pre + "out_proj.weight"], sd[pre + "out_proj.bias"]) + topk_x
    mask = topk_size.log()[:, None, None, :]
    nt = xt.shape[1]
    for i in range(len(model.latent.vit.blocks)):
        pre = f"latent.vit.blocks.{i}."
        h = F.layer_norm(xt, (c,), sd[pre + "norm1.weight"], sd[pre + "norm1.bias"])
        qkv = F.linear(h, sd[pre + "attn.qkv.weight"], sd[pre + "attn.qkv.bias"])
        q, k, v = qkv.view(b, nt, 3, heads, hd).permute(2, 0, 3, 1, 4).unbind(0)
        a = F.scaled_dot_product_attention(q, k, v, attn_mask=mask).transpose(1, 2).reshape(b, nt, c)
        xt = xt + F.linear(a, sd[pre + "attn.proj.weight"], sd[pre + "attn.proj.bias"])
        h = F.layer_norm(xt, (c,), sd[pre + "norm2.weight"], sd[pre + "norm2.bias"])
        h = F.gelu(F.linear(h, sd[pre + "mlp.fc1.weight"], sd[pre + "mlp.fc1.bias"]))
        xt = xt + F.linear(h, sd[pre + "mlp.fc2.weight"], sd[pre + "mlp.fc2.bias"])
    cls = F.layer_norm(xt[:, 0], (c,), sd["latent.vit.norm.weight"], sd["latent.vit.norm.bias"])
    logits = F.linear(cls, sd["head.weight"], sd["head.bias"])
    return logits, topk_idx.numpy()
