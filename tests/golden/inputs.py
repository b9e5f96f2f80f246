"""Seeded synthetic inputs shared by the fixture generator, the tests and the bench.

Inputs are a pure function of (seed, shape): numpy's PCG64 stream, so the GPU
box regenerates exactly the arrays the fixtures were computed from, without
storing them.  Distributions follow the canonical model's routing inputs:
tokens ~ N(0, 1); metric features ~ N(0, 1.3^2) (the output scale of a
Xavier-uniform Linear(384, 64) head on N(0, 1) tokens), stored in float16 as
fp16 autocast produces them.
"""
from __future__ import annotations

import numpy as np

METRIC_SCALE = 1.3


def routing_inputs(seed, batch, grid, channels, metric_dim=64, layers=6,
                   metric_dtype=np.float16, x_dtype=np.float32):
    """x [B, 1+H*W, C] and metrics [L, B, 1+H*W, Cm] (CLS row first)."""
    rng = np.random.default_rng(seed)
    t = 1 + int(grid[0]) * int(grid[1])
    x = rng.standard_normal((batch, t, channels), dtype=np.float32)
    metrics = rng.standard_normal((layers, batch, t, metric_dim), dtype=np.float32)
    metrics = (metrics * np.float32(METRIC_SCALE)).astype(metric_dtype)
    return x.astype(x_dtype), metrics


def canonical_r_list(grid, layers=6, lambda_local=2.0):
    """The model's per-layer merge budget: total = P*(lambda-1)/lambda spread
    by parse_r (model.py:752-754, :407, :546-551)."""
    p = int(grid[0]) * int(grid[1])
    total = int(p * (lambda_local - 1) / lambda_local)
    default_r = total // max(layers, 1)
    r_list = [default_r] * layers
    r_list[-1] += total - sum(r_list)
    return r_list


def attention_inputs(seed, batch, tokens, heads, head_dim, std=0.02, dtype=np.float16):
    """q, k, v [B, N, H, D] ~ N(0, std^2) and a per-key bias [B, N] ~ N(0, std^2)."""
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal((batch, tokens, heads, head_dim), dtype=np.float32) * np.float32(std)
               for _ in range(3))
    bias = rng.standard_normal((batch, tokens), dtype=np.float32) * np.float32(std)
    return q.astype(dtype), k.astype(dtype), v.astype(dtype), bias.astype(dtype)
