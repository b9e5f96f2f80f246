"""CPU port of the mergenet_small_cls inference forward (timed CPU baseline).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Used by ``bench.py``
for its CPU-baseline leg and ``--impl reference`` arm: the reference itself
cannot run on a host without its GPU-only FlashAttention and without timm, so
this port restates its forward (opentome/models/mergenet/model.py:1141-1222)
on the host cores in float32: torch CPU for the dense layers, the windowed
attention of bias_local_attn.py:679-724 as a banded softmax, the numpy routing
oracle for the six merge layers and the carrier block, SDPA-equivalent
cross- and latent attention.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import routing as R


def _band_attention(q, k, v, window, cls_global):
    # q/k/v [B, H, N, D]
    n = q.shape[-2]
    s = (q @ k.transpose(-1, -2)) / q.shape[-1] ** 0.5
    pos = torch.arange(n)
    allowed = (pos[:, None] - pos[None, :]).abs() <= window
    if cls_global:
        allowed[0] = True
    s = s.masked_fill(~allowed, float("-inf"))
    return torch.softmax(s, -1) @ v


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
    route = R.route_and_gather(x.numpy(), [m.numpy() for m in metrics], model.r_list, geom)
    topk_x = torch.from_numpy(route["topk_x"])
    topk_size = torch.from_numpy(route["topk_size"])
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
    return logits, np.asarray(route["topk_idx"])
