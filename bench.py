#!/usr/bin/env python
"""Headline benchmark: fused bf16 matmul + top-k.

10,000,000 items x d=128 from a mixture of 1,024 Gaussian centres (centres
N(0,1), within-cluster sigma 0.15, L2-normalised, bf16), 1,024 queries sampled
the same way, k=100, inner-product score. One step = one query batch against
the whole corpus. With N GPUs (torchrun, one process per GPU) the corpus is
row-sharded (strong scaling: the corpus and batch are fixed); each step is the
local fused top-k, an NCCL all-gather of the per-shard lists and the merge.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line. ``value`` is queries/s with the inputs resident in
HBM, timed with CUDA events, max over ranks; ``e2e`` is the same metric through
the public op with the query batch copied from pinned host memory and the
(ids, scores) copied back every step. ``--impl reference`` times the
reference's CPU path for this workload (the oracle port of FullScanKNN:
fp32 matmul + top-k with ties to the lower id) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "queries/s @10M items d=128 k=100 at 1/2/4/8 B200; roofline %; recall vs ref"
N_ITEMS, DIM, BATCH, K = 10_000_000, 128, 1024, 100
N_CENTRES, SIGMA = 1024, 0.15
BLOCK_ROWS = 1 << 20  # corpus generated in seeded blocks: identical for every world size


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--n-items", type=int, default=N_ITEMS)
    p.add_argument("--batch", type=int, default=BATCH)
    p.add_argument("--k", type=int, default=K)
    p.add_argument("--cpu-sample", type=int, default=16, help="queries in the CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


# ---------------------------------------------------------------------------
# synthetic data (seeded, generated on the device)
# ---------------------------------------------------------------------------
def centres(device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(0)
    return torch.randn(N_CENTRES, DIM, generator=g, device=device)


def mixture_block(cent: torch.Tensor, rows: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device=cent.device).manual_seed(seed)
    c = torch.randint(0, cent.shape[0], (rows,), generator=g, device=cent.device)
    x = cent[c] + SIGMA * torch.randn(rows, DIM, generator=g, device=cent.device)
    x = x / x.norm(dim=1, keepdim=True).clamp_min(1e-8)
    return x.to(torch.bfloat16)


def corpus_rows(cent: torch.Tensor, start: int, end: int, n_total: int) -> torch.Tensor:
    """Rows [start, end) of the global corpus, assembled from its seeded blocks."""
    out = torch.empty((end - start, DIM), dtype=torch.bfloat16, device=cent.device)
    b0, b1 = start // BLOCK_ROWS, (end - 1) // BLOCK_ROWS if end > start else -1
    for b in range(b0, b1 + 1):
        lo, hi = b * BLOCK_ROWS, min((b + 1) * BLOCK_ROWS, n_total)
        blk = mixture_block(cent, hi - lo, 1000 + b)
        s, e = max(lo, start), min(hi, end)
        out[s - start : e - start] = blk[s - lo : e - lo]
    return out


def queries(cent: torch.Tensor, b: int) -> torch.Tensor:
    return mixture_block(cent, b, 7)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.file.name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference CPU path, on a bounded sample
# ---------------------------------------------------------------------------
def host_copy(q_dev: torch.Tensor, x_dev: torch.Tensor, sample: int):
    """fp32 host copies of the corpus and of the first ``sample`` queries."""
    import numpy as np

    xs = [x_dev[lo : lo + BLOCK_ROWS].float().cpu().numpy() for lo in range(0, x_dev.shape[0], BLOCK_ROWS)]
    return q_dev[:sample].float().cpu().numpy(), np.concatenate(xs, axis=0)


def cpu_baseline(q_host, x_host, k: int):
    """One timed run of the oracle port on the host cores → (queries/s, seconds, ids, scores)."""
    from oracle.dense import dense_topk as oracle_dense_topk

    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.perf_counter()
    ref_i, ref_s = oracle_dense_topk(q_host, x_host, k, item_chunk=1 << 20, query_batch=q_host.shape[0])
    dt = time.perf_counter() - t0
    return q_host.shape[0] / dt, dt, ref_i, ref_s


def reference_arm(args):
    """--impl reference: the reference CPU path (oracle port) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    cent = centres(dev)
    x = corpus_rows(cent, 0, args.n_items, args.n_items)
    q = queries(cent, args.batch)
    cores = os.cpu_count() or 1
    q_host, x_host = host_copy(q, x, args.cpu_sample)
    del x
    vals = []
    for i in range(args.warmup + args.steps):
        v, dt, _, _ = cpu_baseline(q_host, x_host, args.k)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "queries/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "dtype": "f32",
        "data": "synthetic",
        "config": config_dict(args),
        "cpu_baseline": {
            "value": value, "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"{args.cpu_sample} queries x full {args.n_items}-item corpus per step",
        },
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(args) -> dict:
    return {
        "workload": "fused bf16 matmul-topk (BASELINE config 2)",
        "n_items": args.n_items,
        "dim": DIM,
        "batch": args.batch,
        "k": args.k,
        "corpus": f"{N_CENTRES}-centre Gaussian mixture, sigma {SIGMA}, L2-normalised, bf16",
        "parallelism": f"row-shard x{args.gpus} + NCCL all-gather",
        "l2": "no flush: the corpus (2.56 GB, or its shard) is larger than L2 (126 MB)",
    }


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from retrieve_b200 import _lib
    from retrieve_b200.shard import ShardedDenseTopK, shard_bounds

    lib = _lib.lib()
    n, b, k = args.n_items, args.batch, args.k
    cent = centres(dev)
    lo, hi = shard_bounds(n, world, rank)
    x = corpus_rows(cent, lo, hi, n)
    q = queries(cent, b)
    index = ShardedDenseTopK(x, lo, k)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up
    for _ in range(args.warmup):
        index.search(q)
    torch.cuda.synchronize()
    barrier()

    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(local)
    sampler.start()
    # device-resident timed region, with the dominant kernel timed per step
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, c in kev:  # torch creates the event handle on first record
        a.record(stream)
        c.record(stream)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        lib.rb_set_profile_events(kev[i][0].cuda_event, kev[i][1].cuda_event)
        index.search(q)
    e1.record(stream)
    lib.rb_set_profile_events(None, None)
    torch.cuda.synchronize()
    barrier()
    t_ms = e0.elapsed_time(e1)
    kern_ms = statistics.mean(a.elapsed_time(c) for a, c in kev)

    # end to end through the public op: pinned host query batch in, results out
    q_host = q.cpu().pin_memory()
    ids_host = torch.empty((b, k), dtype=torch.int64).pin_memory()
    sc_host = torch.empty((b, k), dtype=torch.float32).pin_memory()
    q_dev = torch.empty_like(q)
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        q_dev.copy_(q_host, non_blocking=True)
        ids, sc = index.search(q_dev)
        ids_host.copy_(ids, non_blocking=True)
        sc_host.copy_(sc, non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    e2e_ms = f0.elapsed_time(f1)

    times = torch.tensor([t_ms, e2e_ms, kern_ms], device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, kern_ms = times.tolist()
    value = b * args.steps / (t_ms / 1e3)
    e2e_value = b * args.steps / (e2e_ms / 1e3)

    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = peaks.get("bf16_tflops_sustained")
    peak_note = "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
    if peak is None:
        peak, peak_note = 1400.0, "fallback (sustained 1.4 PFLOP/s)"
    flops = 2.0 * b * (hi - lo) * DIM
    achieved = flops / (kern_ms / 1e3) / 1e12
    traffic = None
    prof = ROOT / "profiles" / "dense_scan_c2_traffic.json"
    if prof.exists():
        tr = json.loads(prof.read_text())
        traffic = tr.get("bytes_per_launch_scaled", {}).get(str(world))

    launches = index.launches_per_search(b) * args.steps

    line = {
        "metric": METRIC,
        "value": value,
        "unit": "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": config_dict(args),
        "e2e": {
            "value": e2e_value,
            "unit": "queries/s",
            "h2d_bytes_per_step": q_host.numel() * q_host.element_size(),
            "d2h_bytes_per_step": ids_host.numel() * 8 + sc_host.numel() * 4,
        },
        "roofline": {
            "bound": "tensor",
            "kernel": "dense_scan_kernel (full-corpus pass)",
            "achieved": achieved,
            "peak": peak,
            "peak_source": peak_note,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "traffic": traffic,
            "kernel_ms": kern_ms,
        },
        "gpu_launches": launches,
        "clocks": clocks,
    }

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        q_host, x_host = host_copy(q, x, args.cpu_sample)
        v, dt, ref_i, ref_s = cpu_baseline(q_host, x_host, k)
        ours_i, _ = index.search(q[: args.cpu_sample])
        from oracle.dense import recall_at_k

        line["cpu_baseline"] = {
            "value": v, "unit": "queries/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{args.cpu_sample} queries x full {n}-item corpus ({dt:.1f} s)",
        }
        line["recall_vs_ref"] = recall_at_k(ours_i.cpu().numpy(), ref_i)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
