#!/usr/bin/env python
"""Headline benchmark: fused bf16 matmul + top-k.

10,000,000 items x d=128 from a mixture of 1,024 Gaussian centres (centres
N(0,1), within-cluster sigma 0.15, L2-normalised, bf16), 1,024 queries sampled
the same way, k=100, inner-product score. One step = one query batch against
the whole corpus. With N GPUs (torchrun, one process per GPU) the corpus is
row-sharded (strong scaling: the corpus and batch are fixed); each step is the
shard sample, an NCCL all-gather of the samples (the shared threshold seed),
the local fused top-k, an all-gather of the per-shard results and the merge.
The step runs as one CUDA graph (retrieve_b200.shard.GraphedSearch), captured
after the warm-up searches.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line. ``value`` is queries/s with the inputs resident in
HBM, timed with CUDA events, max over ranks; ``e2e`` is the same metric through
the public op with the query batch copied from pinned host memory and the
(ids, scores) copied back every step. ``--impl reference`` times the
reference's CPU path for this workload on the host cores: its own FullScanKNN
(fp32 torch matmul + topk) from the reference package installed under
baseline/_ref, or the oracle's numpy restatement of it when that is absent.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
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
    p.add_argument("--cpu-sample", type=int, default=256,
                   help="queries in the CPU-baseline sample of this arm (about 10 s of host work)")
    p.add_argument("--ref-sample", type=int, default=32,
                   help="queries per step of --impl reference (each step a bounded sample)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--reference-device", choices=("cpu", "cuda"), default="cpu",
                   help="--impl reference: the reference's CPU path (FullScanKNN on the host cores, the "
                        "default) or its own GPU path (PostfilterKNN: cuBLAS fp16 scores + masked_topk)")
    p.add_argument("--exchange", choices=("nccl", "peer"), default="nccl",
                   help="the sharded search's two all-gathers: NCCL, or stores into the peers' memory")
    p.add_argument("--no-configs", action="store_true",
                   help="skip the records of configs 3, 4, 5 and the IVF search that follow the headline at N=1")
    p.add_argument("--workload", choices=("c2", "c3", "c4", "c5", "ivf", "ops"), default="c2",
                   help="c2 (default, the headline); c3/c4/c5 and ops: one-GPU measurements of the other configs "
                        "and of every other kernel")
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
    """Samples this rank's GPU SM clock and clock-event reasons through NVML
    (read-only queries) from a thread, every few milliseconds, while running."""

    REASONS = {  # NVML clocks-event reason bits
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, device: torch.device, interval_s: float = 0.002):
        self.interval = interval_s
        self.samples: list[tuple[float, float, int]] = []
        self.error = None
        self._stop = None
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception as exc:  # NVML missing or the device not found
            self.nvml = None
            self.error = f"nvml unavailable: {type(exc).__name__}"

    def _read(self):
        nv = self.nvml
        sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
        reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        self.samples.append((float(sm), float(mx), int(reasons)))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._read()
            except Exception as exc:
                self.error = f"nvml read failed: {type(exc).__name__}"
                return
            self._stop.wait(self.interval)

    def start(self):
        import threading

        if self.nvml is None:
            return
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def stop(self) -> list:
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        return list(self.samples)

    @classmethod
    def summary(cls, per_rank: list[tuple[list, str | None]]) -> dict:
        sm, mx, bits, errors = [], [], 0, []
        for samples, err in per_rank:
            if err:
                errors.append(err)
            for a, b, r in samples:
                sm.append(a)
                mx.append(b)
                bits |= r
        reasons = sorted(name for bit, name in cls.REASONS.items() if bits & bit)
        out = {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons + errors,
            "samples": len(sm),
            "source": "NVML, every rank's GPU, sampled every 2 ms during the timed regions",
        }
        return out


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own CPU torch path (FullScanKNN from the
# reference package installed under baseline/_ref), else the oracle port
# ---------------------------------------------------------------------------
REF_SITE = ROOT / "baseline" / "_ref"


def host_copy(q_dev: torch.Tensor, x_dev: torch.Tensor, sample: int):
    """fp32 host copies (torch tensors) of the corpus and of the first ``sample`` queries."""
    xs = torch.empty((x_dev.shape[0], x_dev.shape[1]), dtype=torch.float32)
    for lo in range(0, x_dev.shape[0], BLOCK_ROWS):
        xs[lo : lo + BLOCK_ROWS] = x_dev[lo : lo + BLOCK_ROWS].float().cpu()
    return q_dev[:sample].float().cpu(), xs


def reference_cpu_search(x_host: torch.Tensor, k: int):
    """``(search, kind)``: ``search(q) -> (ids, scores)`` over the fp32 host corpus on every
    host core. ``kind`` "reference" runs the reference's ``FullScanKNN``
    (retrieve/src/retrieve/modules/knn.py:125-170: ``query @ item_embs.t()`` then
    ``torch.topk``) from its installed package, 32 queries per forward call; "port" runs the
    oracle's numpy restatement of the same path when that package is absent."""
    torch.set_num_threads(os.cpu_count() or 1)
    if (REF_SITE / "retrieve").is_dir():
        if str(REF_SITE) not in sys.path:
            sys.path.insert(0, str(REF_SITE))
        from retrieve.modules.knn import FullScanKNN

        module = FullScanKNN(k=k)
        module.register_index(x_host)

        def search(q: torch.Tensor):
            outs = [module(q[i : i + 32]) for i in range(0, q.shape[0], 32)]
            return torch.cat([o[0] for o in outs]), torch.cat([o[1] for o in outs])

        return search, "reference"
    from oracle.dense import dense_topk as oracle_dense_topk

    xn = x_host.numpy()

    def search_port(q: torch.Tensor):
        ids, sc = oracle_dense_topk(q.numpy(), xn, k, item_chunk=1 << 20, query_batch=q.shape[0])
        return torch.from_numpy(ids), torch.from_numpy(sc)

    return search_port, "port"


def cpu_baseline(q_host: torch.Tensor, x_host: torch.Tensor, k: int):
    """One timed run of the reference CPU path on the host cores →
    (queries/s, seconds, ids, kind)."""
    search, kind = reference_cpu_search(x_host, k)
    t0 = time.perf_counter()
    ref_i, _ = search(q_host)
    dt = time.perf_counter() - t0
    return q_host.shape[0] / dt, dt, ref_i.numpy(), kind


def reference_gpu_arm(args):
    """--impl reference --reference-device cuda: the reference's own GPU path for this search,
    ``PostfilterKNN`` (retrieve/src/retrieve/modules/knn.py:23-76: the corpus cast to fp16 and
    pre-transposed, cuBLAS ``torch.mm(..., out_dtype=float32)`` over every item, then
    ``masked_topk``'s two-level top-k) from its installed package, on the same corpus and query
    batch, the whole batch per call, CUDA events around each call. Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if not (REF_SITE / "retrieve").is_dir():
        print(json.dumps({"impl": "reference", "unavailable": "the reference package is not installed under "
                          "baseline/_ref"}), flush=True)
        return
    if str(REF_SITE) not in sys.path:
        sys.path.insert(0, str(REF_SITE))
    from retrieve.modules.knn import PostfilterKNN

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    cent = centres(dev)
    x = corpus_rows(cent, 0, args.n_items, args.n_items)
    q = queries(cent, args.batch)
    module = PostfilterKNN(k=args.k, backend="torch")
    module.register_index(x)
    del x
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        module(q)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, b in ev:
        a.record()
        module(q)
        b.record()
    torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    value = args.batch / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "fp16 scores in fp32", "data": "synthetic", "config": config_dict(args),
        "reference_device": "cuda",
        "reference_path": "PostfilterKNN (torch backend): cuBLAS fp16 x fp16 -> fp32 [B, N] scores, masked_topk",
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def reference_arm(args):
    """--impl reference: the reference's CPU path on the host cores, rank 0 only."""
    if getattr(args, "reference_device", "cpu") == "cuda":
        reference_gpu_arm(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    cent = centres(dev)
    x = corpus_rows(cent, 0, args.n_items, args.n_items)
    q = queries(cent, args.batch)
    cores = os.cpu_count() or 1
    q_host, x_host = host_copy(q, x, args.ref_sample)
    del x
    search, kind = reference_cpu_search(x_host, args.k)
    vals = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        search(q_host)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            vals.append(q_host.shape[0] / dt)
    value = statistics.median(vals)
    what = ("the reference's FullScanKNN (torch matmul + topk, fp32)" if kind == "reference"
            else "the oracle port of FullScanKNN (numpy)")
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
            "value": value, "unit": "queries/s", "cores": cores, "kind": kind,
            "sample": f"{args.ref_sample} queries x full {args.n_items}-item corpus per step, {what}",
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
        "parallelism": f"row-shard x{args.gpus}, shared seed; 2 all-gathers per step "
                       f"({'stores into peer memory' if args.exchange == 'peer' else 'NCCL'}); "
                       "one CUDA graph per step",
        "l2": "no flush: the corpus (2.56 GB, or its shard) is larger than L2 (126 MB)",
    }


def main():
    args = parse_args()
    if args.workload != "c2":
        from bench_configs import run_workload

        run_workload(args)
        return
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

        # NCCL's communicator lines (ranks per communicator) stay in the log
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from retrieve_b200 import _lib
    from retrieve_b200.shard import GraphedSearch, ShardedDenseTopK, shard_bounds

    lib = _lib.lib()
    n, b, k = args.n_items, args.batch, args.k
    cent = centres(dev)
    lo, hi = shard_bounds(n, world, rank)
    x = corpus_rows(cent, lo, hi, n)
    q = queries(cent, b)
    index = ShardedDenseTopK(x, lo, k, n_total=n, exchange=args.exchange)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up through the plain (uncaptured) search
    for _ in range(args.warmup):
        index.search(q)
    torch.cuda.synchronize()
    barrier()

    # value: K back-to-back replays of the one-search graph (GraphedSearch, the
    # public API's captured search), inputs resident in HBM, nothing else in it
    stream = torch.cuda.current_stream(dev)
    graphed = GraphedSearch(index, q, warmup=1)
    # kernel time: K eager searches with an event pair around each full-corpus pass,
    # recorded on the stream the pass runs on (timed in a region of its own, after
    # value's; event nodes inside a graph slowed the replay, eager records do not
    # touch the pass itself)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for ka, kb in kev:
        ka.record(stream)
        kb.record(stream)
    for _ in range(args.warmup):
        graphed.replay()
    torch.cuda.synchronize()
    barrier()

    sampler = ClockSampler(dev)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        graphed.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    t_ms = e0.elapsed_time(e1)

    barrier()
    torch.cuda.synchronize()
    i0, i1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    i0.record(stream)
    for ka, kb in kev:
        lib.rb_set_profile_events(ka.cuda_event, kb.cuda_event)
        index.search(graphed.query)
    lib.rb_set_profile_events(None, None)
    i1.record(stream)
    torch.cuda.synchronize()
    barrier()
    inst_ms = i0.elapsed_time(i1)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)

    # end to end through the public API: pinned host query batch in, results out
    q_host = q.cpu().pin_memory()
    ids_host = torch.empty((b, k), dtype=torch.int64).pin_memory()
    sc_host = torch.empty((b, k), dtype=torch.float32).pin_memory()
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        ids, sc = graphed.search(q_host)
        ids_host.copy_(ids, non_blocking=True)
        sc_host.copy_(sc, non_blocking=True)
    f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    samples = sampler.stop()
    e2e_ms = f0.elapsed_time(f1)
    per_rank = [(samples, sampler.error)]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, (samples, sampler.error))
        per_rank = gathered
    clocks = ClockSampler.summary(per_rank)

    times = torch.tensor([t_ms, e2e_ms, kern_ms, inst_ms], device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, kern_ms, inst_ms = times.tolist()
    value = b * args.steps / (t_ms / 1e3)
    e2e_value = b * args.steps / (e2e_ms / 1e3)

    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    # The scan runs for milliseconds at a time inside a region of well under a
    # second, at the clocks sampled below: its denominator is the burst GEMM peak.
    peak = peaks.get("bf16_tflops")
    peak_note = "measured (MEASURED_PEAKS.json bf16_tflops, the burst figure)"
    if peak is None:
        peak, peak_note = 1590.0, "fallback (burst 1.59 PFLOP/s)"
    peak_sustained = peaks.get("bf16_tflops_sustained")
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
            "frac_of_sustained": achieved / peak_sustained if peak_sustained else None,
            "traffic": traffic,
            "kernel_ms": kern_ms,
            "kernel_ms_source": "CUDA events recorded on the pass's stream around the full-corpus pass of each "
                                "of K eager searches (a region of its own), mean over searches, max over ranks",
            "instrumented_ms_per_step": inst_ms / args.steps,
        },
        "gpu_launches": launches,
        "clocks": clocks,
    }

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        q_host, x_host = host_copy(q, x, args.cpu_sample)
        v, dt, ref_i, kind = cpu_baseline(q_host, x_host, k)
        del x_host
        ours_i, _ = index.search(q[: args.cpu_sample])
        from oracle.dense import recall_at_k

        line["cpu_baseline"] = {
            "value": v, "unit": "queries/s", "cores": os.cpu_count(), "kind": kind,
            "sample": f"{args.cpu_sample} queries x full {n}-item corpus ({dt:.1f} s)",
        }
        line["recall_vs_ref"] = recall_at_k(ours_i.cpu().numpy(), ref_i)
    graphed.release()
    if world > 1:
        index.close()  # the peer exchange buffers (collective; nothing with NCCL)
    if world == 1 and not args.no_configs:
        # the other configurations, one GPU each, after the headline's inputs are freed
        from bench_configs import measure_configs

        del index, x, q
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        line["configs"] = measure_configs(args, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
