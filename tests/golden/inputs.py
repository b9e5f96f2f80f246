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


def model_weights(shapes, seed=0):
    """A full set of model weights as a pure function of (seed, parameter
    name, shape): {name: float32 array}.  Each tensor draws from its own
    PCG64 stream keyed by a CRC of its name, so the set does not depend on
    the order of the names.  1-D norm weights ~ 1 + N(0, 0.05^2); biases,
    position embedding and CLS token ~ N(0, 0.02^2); weight matrices and the
    patch kernel ~ N(0, 1 / fan_in).  The recovery out-projection is not
    zero here, so it takes part in every comparison."""
    import zlib
    out = {}
    for name, shape in shapes.items():
        rng = np.random.default_rng([int(seed), zlib.crc32(name.encode())])
        shape = tuple(int(v) for v in shape)
        z = rng.standard_normal(shape, dtype=np.float32)
        leaf = name.rsplit(".", 1)[-1]
        if len(shape) == 1 and "norm" in name and leaf == "weight":
            w = 1.0 + 0.05 * z
        elif leaf == "bias" or leaf in ("pos_embed", "cls_token"):
            w = 0.02 * z
        else:
            fan_in = int(np.prod(shape[1:])) if len(shape) > 1 else shape[0]
            w = z / np.sqrt(fan_in)
        out[name] = w.astype(np.float32)
    return out


def model_images(seed, batch, size=224):
    """Synthetic N(0, 1) images [B, 3, size, size]."""
    rng = np.random.default_rng([int(seed), 224])
    return rng.standard_normal((batch, 3, size, size), dtype=np.float32)
