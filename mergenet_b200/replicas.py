"""Batch-sharded replicas: the multi-GPU plumbing around the hot path.

Every image's routing is independent except through ThreTopK's batch-global
range, which is per launch and so per GPU: each rank runs a complete batch,
and nothing crosses GPUs on the hot path.  The only collectives are for
reporting: the maximum step time over ranks and a gather of the logits for
checking (the reference trainer's SUM/MAX reductions and concat_all_gather,
trainer/classification/in1k_trainer.py:2847-2850, :2902-2913).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def world():
    """(world_size, rank) of the default process group, or (1, 0)."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def shard_bounds(global_batch, world_size, rank):
    """[start, end) of this rank's images when a global batch is split."""
    per, extra = divmod(int(global_batch), int(world_size))
    start = rank * per + min(rank, extra)
    return start, start + per + (1 if rank < extra else 0)


def max_over_ranks(seconds, device=None):
    """Largest per-rank device time (the step is as slow as its slowest GPU)."""
    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    if world()[0] > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_logits(logits):
    """All ranks' logits, concatenated in rank order (every rank receives it)."""
    n, _ = world()
    if n == 1:
        return logits
    parts = [torch.empty_like(logits) for _ in range(n)]
    dist.all_gather(parts, logits.contiguous())
    return torch.cat(parts, 0)
