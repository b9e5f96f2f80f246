"""The replica plumbing on two gloo ranks (CPU): shard bounds, the timing MAX
and the logits gather that bench.py uses under torchrun."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mergenet_b200.replicas import gather_logits, max_over_ranks, shard_bounds, world as w
        assert w() == (world, rank)
        t = max_over_ranks(0.5 + rank)  # rank 1 is the slow one
        logits = torch.full((3, 4), float(rank))
        allg = gather_logits(logits)
        q.put((rank, t, allg.tolist(), shard_bounds(10, world, rank)))
    finally:
        dist.destroy_process_group()


def test_two_rank_replicas():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out.sort()
    for rank, t, allg, bounds in out:
        assert t == pytest.approx(1.5)
        assert allg == [[0.0] * 4] * 3 + [[1.0] * 4] * 3
    assert [o[3] for o in out] == [(0, 5), (5, 10)]


def test_shard_bounds_cover_the_batch():
    from mergenet_b200.replicas import shard_bounds
    for total in (0, 1, 7, 256, 1000):
        for n in (1, 2, 3, 8):
            spans = [shard_bounds(total, n, r) for r in range(n)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
