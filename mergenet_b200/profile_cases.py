"""Small, fixed workloads of the library's kernels, for profilers.

    python -m mergenet_b200.profile_cases attention [--batch 128] [--iters 2]
    python -m mergenet_b200.profile_cases routing   [--batch 128] [--iters 2]
    python -m mergenet_b200.profile_cases training  [--batch 128] [--iters 2]

Each case runs ``iters`` identical iterations on ``cuda:0`` with seeded
synthetic inputs of the mergenet_small_cls shapes (224x224 images, patch 8:
785 tokens, 6 heads of 64, 393 latent tokens) and prints the status words, so
a profiler can skip the first iteration's launches and capture the second's.

* ``attention``: windowed local attention with the CLS row (packed qkv
  [B, 785, 1152] fp16, window 16), latent attention over 393 tokens with a
  per-key log-size bias, and the 393 x 785 recovery cross-attention (the
  last two on the warp-specialised kernel).
* ``routing``: the fused six-layer routing and carrier gather on x_embed
  [B, 785, 384] fp32 and metrics [6, B, 785, 64] fp16.
* ``gemm``: the MLP GEMMs of one local block on B x 785 token rows: fc1 with
  the GELU epilogue (384 -> 1536), then fc2 (1536 -> 384).
* ``training``: one training-mode merge layer (DTEMMergeBlock, x [B, 785,
  384] fp32, metric 64, r = 65, the strided parity grouping) forward and
  backward: the drop-in score, select and transport kernels and their
  gradients.
"""
from __future__ import annotations

import argparse

import torch


def attention(batch, iters):
    from . import attention as A
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = (torch.randn(batch, 785, 1152, device=dev, generator=g) * 0.5).half()
    lat = (torch.randn(batch, 393, 1152, device=dev, generator=g) * 0.5).half()
    log_size = (torch.rand(batch, 393, device=dev, generator=g) + 0.1).log()
    q = torch.randn(batch, 393, 6, 64, device=dev, generator=g).half()
    kv = torch.randn(batch, 785, 2, 6, 64, device=dev, generator=g).half()
    for _ in range(iters):
        A.local_attention_packed(qkv, 6, 16, cls_global=True)
        A.local_attention_packed(lat, 6, -1, cls_global=False, bias=log_size)
        A.cross_attention(q, kv[:, :, 0], kv[:, :, 1], out_dtype=torch.float32)
    torch.cuda.synchronize()
    print("attention status", A.attention_status(dev))


def routing(batch, iters):
    from .routing import RoutePlan
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(batch, 785, 384, device=dev, generator=g)
    metrics = (torch.randn(6, batch, 785, 64, device=dev, generator=g) * 1.3).half()
    plan = RoutePlan((28, 28), 3.0, [65, 65, 65, 65, 65, 67], device=dev)
    res = None
    for _ in range(iters):
        res = plan(x, metrics)
    torch.cuda.synchronize()
    print("routing status", int(res.status.item()))


def gemm(batch, iters):
    from .linear import gemm_status, linear_f16
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    h = torch.randn(batch * 785, 384, device=dev, generator=g).half()
    w1 = (torch.randn(1536, 384, device=dev, generator=g) * 0.05).half()
    b1 = torch.zeros(1536, device=dev, dtype=torch.float16)
    w2 = (torch.randn(384, 1536, device=dev, generator=g) * 0.025).half()
    b2 = torch.zeros(384, device=dev, dtype=torch.float16)
    for _ in range(iters):
        f = linear_f16(h, w1, b1, gelu=True)
        linear_f16(f, w2, b2)
    torch.cuda.synchronize()
    print("gemm status", gemm_status(dev))


def training(batch, iters):
    from .dtem import make_merge_block
    from .routing import check_status  # noqa: F401  (the library must load)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    block = make_merge_block((28, 28), 3.0, device=dev).train()
    block._tome_info.update({"train_grouping": "alternating_per_layer_fast", "merge_layer_index": 1})
    x = torch.randn(batch, 785, 384, device=dev, generator=g).requires_grad_(True)
    metric = torch.randn(batch, 785, 64, device=dev, generator=g).requires_grad_(True)
    size = torch.ones(batch, 785, 1, device=dev)
    gx = torch.randn(batch, 785, 384, device=dev, generator=g)
    gs = torch.randn(batch, 785, 1, device=dev, generator=g)
    for _ in range(iters):
        block._tome_info["token_center"] = None
        xo, so, _, _, _ = block._merge_train(x, size, 65, 785, {"metric": metric})
        torch.autograd.backward([xo, so], [gx, gs])
    torch.cuda.synchronize()
    print("training grads finite", bool(torch.isfinite(x.grad).all() and torch.isfinite(metric.grad).all()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["attention", "routing", "gemm", "training"])
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--iters", type=int, default=2)
    args = ap.parse_args()
    {"attention": attention, "routing": routing, "gemm": gemm, "training": training}[args.case](args.batch,
                                                                                               args.iters)


if __name__ == "__main__":
    main()
