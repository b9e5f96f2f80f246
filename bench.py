#!/usr/bin/env python3
"""Benchmark: mergenet_small_cls fp16 inference images/sec on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference]

One step = one full forward of the canonical model (224x224, patch 8, routing
784 -> 392 carriers) over B synthetic N(0,1) images per GPU, random init
(seed 0).  Multi-GPU runs are batch-sharded replicas (launched by torchrun, one
rank per GPU, NCCL only for the timing max and the logits check): per-GPU work
is fixed, so scaling is weak.  Prints ONE JSON line on rank 0.

--impl reference times the reference path's CPU port (the reference needs
FlashAttention on a GPU and timm, neither usable on the host) on this box's
host cores: the float32 forward of oracle/model_cpu.py over a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import tempfile
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "images/sec mergenet_small_cls fp16 B=256/GPU"
IMG = 224
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum, one ncu capture
# of a B=128 launch) of the windowed attention kernel with its CLS row and of
# the latent attention kernel, per image; the traffic grows in proportion to
# the batch
TRAFFIC_LOCAL_ATTN = 313.3e6 / 128
TRAFFIC_LATENT_ATTN = 136.3e6 / 128
PEAKS = ROOT / "MEASURED_PEAKS.json"


def _peaks():
    try:
        d = json.loads(PEAKS.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        # the raw samples go to $MN_CLOCKS_DIR (default: the system temp dir)
        out = Path(os.environ.get("MN_CLOCKS_DIR", tempfile.gettempdir()))
        self.path = out / f"mergenet_b200_clocks_gpu{index}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(1.0)  # let nvidia-smi attach before the timed region starts
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        try:
            rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
            sm = [float(r[0]) for r in rows]
            reasons = set()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for r in rows:
                for name, val in zip(names, r[3:7]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][1]), "samples": len(rows),
                    "reasons": sorted(reasons)}
        except Exception:
            return None


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _time_kernel(fn, stream, iters=10):
    """Average duration of fn (launching on `stream`) with CUDA events."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record(stream)
        for _ in range(iters):
            fn()
        e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters / 1e3


def cpu_port_rate(model, seconds=12.0, batch=2, threads=None):
    """Images/sec of the float32 CPU port on the host cores (bounded sample)."""
    from oracle import model_cpu, routing
    torch.set_num_threads(threads or os.cpu_count() or 1)
    cpu_model = model
    geom = routing.Geometry(model.grid, model.spatial_radius)
    g = torch.Generator().manual_seed(1)
    images = torch.randn(batch, 3, IMG, IMG, generator=g)
    done, t0 = 0, time.perf_counter()
    while True:
        model_cpu.forward(cpu_model, images, geom)
        done += batch
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return done / dt, done, dt


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    from mergenet_b200.model import ForwardGraph, MergeNetSmall
    model = MergeNetSmall().init_weights(0)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle import model_cpu, routing
    geom = routing.Geometry(model.grid, model.spatial_radius)
    g = torch.Generator().manual_seed(1)
    images = torch.randn(args.ref_sample, 3, IMG, IMG, generator=g)
    for _ in range(args.warmup):
        model_cpu.forward(model, images, geom)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model_cpu.forward(model, images, geom)
    dt = time.perf_counter() - t0
    value = args.ref_sample * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/sec", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "mergenet_small_cls forward, 224x224, CPU port of the reference path",
                   "sample_images_per_step": args.ref_sample},
        "cpu_baseline": {"value": value, "unit": "images/sec", "cores": threads, "kind": "port",
                         "sample": f"{args.ref_sample} images per step x {args.steps} steps, float32 CPU port "
                                   "(oracle/model_cpu.py)"},
        "e2e": {"value": value, "unit": "images/sec", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args):
    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import mergenet_b200
    from mergenet_b200 import _lib
    from mergenet_b200.model import ForwardGraph, MergeNetSmall
    from mergenet_b200.replicas import gather_logits, max_over_ranks

    _lib.lib()
    model = MergeNetSmall().init_weights(0).to(dev).eval()
    B = args.batch
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    images = torch.randn(B, 3, IMG, IMG, device=dev, generator=g)  # 154 MB: larger than L2
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # the forward is captured once as a CUDA graph (after `warmup` eager
    # forwards) and replayed: same kernels, no per-kernel host launch cost
    fwd = ForwardGraph(model, images, warmup=args.warmup)
    for _ in range(args.warmup):
        fwd()
    barrier()
    sampler = ClockSampler(local)
    with sampler:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            logits, aux = fwd()
        end.record(stream)
        barrier()
    t_max = max_over_ranks(start.elapsed_time(end) / 1e3, dev)
    value = world * B * args.steps / t_max
    fwd.check_status()  # fail closed on any device status the timed replays raised

    # end to end through the public call: pinned host images -> device -> logits -> host
    # every step copies its pinned host batch to the device (on a copy stream,
    # overlapping the previous step's forward) and reads its logits back
    host_images = images.cpu().pin_memory()
    host_logits = torch.empty(max(args.steps, args.warmup // 2, 1), B, logits.shape[1], dtype=logits.dtype).pin_memory()
    fwd.run_host_batches([host_images] * max(1, args.warmup // 2), host_logits)
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    fwd.run_host_batches([host_images] * args.steps, host_logits)
    e2.record(stream)
    barrier()
    e2e_value = world * B * args.steps / max_over_ranks(s2.elapsed_time(e2) / 1e3, dev)

    # logits check across ranks (the only data collective): every rank's
    # logits are finite and gathered
    finite = bool(torch.isfinite(gather_logits(logits)).all())

    # roofline of the dominant library kernel, the windowed local attention
    # with its CLS row (attn_tc_kernel<half, 160, window>), and of the latent
    # attention over all 393 carriers with the log-size bias
    nt = 393
    qkv_l = torch.randn(B, nt, 3 * 384, device=dev, dtype=torch.float16) * 0.5
    log_size = torch.rand(B, nt, device=dev).mul_(3.0).log1p_()
    t_attn = _time_kernel(lambda: mergenet_b200.local_attention_packed(qkv_l, 6, -1, cls_global=False,
                                                                         bias=log_size), stream)
    attn_bytes = qkv_l.numel() * 2 + log_size.numel() * 4 + B * nt * 384 * 2  # q,k,v,bias read + o write
    attn_flops = 4 * B * 6 * nt * nt * 64
    peak, peak_kind = _peaks()
    achieved = attn_bytes / t_attn / 1e9
    qkv = torch.randn(B, 785, 3 * 384, device=dev, dtype=torch.float16) * 0.5
    t_local = _time_kernel(lambda: mergenet_b200.local_attention_packed(qkv, 6, 16, cls_global=True), stream)
    local_bytes = qkv.numel() * 2 + B * 785 * 384 * 2  # q, k, v read + o write (fp16)
    local_achieved = local_bytes / t_local / 1e9
    # the routing op on the same shard (routing HBM GB/s)
    x_embed = torch.randn(B, 785, 384, device=dev)
    metrics = (torch.randn(6, B, 785, 64, device=dev) * 1.3).half()
    plan = model._plan(dev)
    t_route = _time_kernel(lambda: plan(x_embed, metrics), stream)
    route_bytes = B * (6 * 785 * 64 * 2 + 785 * 384 * 4 + 393 * 384 * 4 + 785 * 4 * 3 + 392 * 8)

    line = None
    if rank == 0:
        cpu_v, cpu_n, cpu_t = cpu_port_rate(MergeNetSmall().init_weights(0),
                                            seconds=args.cpu_seconds) if world == 1 else (None, 0, 0.0)
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "images/sec", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "mergenet_small_cls forward (config 4): 224x224 images, patch 8, 6 local + "
                                   "6 latent blocks, routing 784->392, fp16 autocast semantics",
                       "global_batch": B * world, "per_gpu_batch": B, "parallelism": f"batch-shard x{world}",
                       "l2": "inputs larger than L2 (154 MB images per step)", "logits_finite": finite},
            "e2e": {"value": e2e_value, "unit": "images/sec", "h2d_bytes_per_step": host_images.numel() * 4,
                    "d2h_bytes_per_step": host_logits[0].numel() * host_logits.element_size(),
                    "overlap": "H2D of step i+1 on a copy stream during step i's forward"},
            "gpu_launches": ForwardGraph.library_launches(model) * args.steps,
            "roofline": {"kernel": "attn_win_persistent_kernel<half> with the CLS row folded in (local attention, "
                                   "window 16, 785 tokens, 6 heads, B=%d)" % B,
                         "bound": "hbm", "achieved": local_achieved, "peak": peak, "unit": "GB/s",
                         "frac": local_achieved / peak, "peak_kind": peak_kind, "traffic": TRAFFIC_LOCAL_ATTN * B,
                         "algorithmic_bytes": local_bytes, "ms_per_launch": t_local * 1e3},
            "latent_attention": {"kernel": "attn_tc_kernel<half,64,full,bias> (393 carriers, 6 heads)",
                                 "ms_per_call": t_attn * 1e3, "algorithmic_bytes": attn_bytes,
                                 "achieved_gbs": achieved, "frac": achieved / peak,
                                 "traffic": TRAFFIC_LATENT_ATTN * B, "tflops": attn_flops / t_attn / 1e12},
            "routing": {"ms_per_call": t_route * 1e3, "algorithmic_bytes": route_bytes,
                        "achieved_gbs": route_bytes / t_route / 1e9, "frac": route_bytes / t_route / 1e9 / peak},
            "cpu_baseline": ({"value": cpu_v, "unit": "images/sec", "cores": os.cpu_count(), "kind": "port",
                              "sample": f"{cpu_n} images in {cpu_t:.1f} s, float32 CPU port (oracle/model_cpu.py)"}
                             if cpu_v is not None else None),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-sample", type=int, default=1)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
