"""One-GPU measurements of the configurations other than the headline, and of
every kernel outside the dense scan, for ``bench.py --workload c3|c4|c5|ops``.

Each prints one JSON line in ``bench.py``'s format (metric, value, unit, config,
roofline with the measured peaks, clocks). Inputs are seeded synthetic data of
the BASELINE configurations' shapes, generated on the device; timing is CUDA
events around W untimed + K timed steps; every input is larger than L2 (or the
step streams more than L2), so no flush is needed.

  c3   attribute-filtered kNN, fp16 10M x 128, 8 Zipf(1.1) attributes, per-item
       64-bit Bloom words (3 hashes), B = 1024, k = 100, predicates of 1-3
       terms at about 1 %, 10 % and 50 % selectivity (Bloom test + exact recheck)
  c4   int8 scoring, 30M x 256 with per-row scales, B = 4096, k = 100
  c5   1-bit pool + rerank, 30M x 512-bit SimHash codes of a d = 128 mixture,
       pool 1000 on the int8 tensor cores, fp16 rerank to k = 100, B = 1024
  ivf  SilverTorch's IVF search: phase 1 (centroid scores + probe top-k) and
       st::search (int8 probe scoring, top-k, dequant) over an int8 table of the
       C2 corpus in cluster-sorted order, 1024 lists, 16 probes, B = 1024, k = 100
  ops  the remaining kernels one by one at representative sizes
"""

from __future__ import annotations

import json
from pathlib import Path
import statistics

import torch

import bench

N_CENTRES, SIGMA = bench.N_CENTRES, bench.SIGMA


def _centres(dim: int, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(0)
    return torch.randn(N_CENTRES, dim, generator=g, device=device)


def _mixture(cent: torch.Tensor, rows: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device=cent.device).manual_seed(seed)
    c = torch.randint(0, cent.shape[0], (rows,), generator=g, device=cent.device)
    x = cent[c] + SIGMA * torch.randn(rows, cent.shape[1], generator=g, device=cent.device)
    return x / x.norm(dim=1, keepdim=True).clamp_min(1e-8)


def _blocks(n: int, fn, block: int = 1 << 20):
    for b, lo in enumerate(range(0, n, block)):
        yield lo, min(lo + block, n), fn(min(lo + block, n) - lo, 1000 + b)


def _time(step, warmup: int, steps: int, kernel: bool = True) -> tuple[float, float | None]:
    """(mean ms per step, mean ms of the step's dominant kernel or None) over K timed
    steps after W warm-ups. Each step is bracketed by CUDA events on the launching
    stream; with ``kernel`` the library's profiling hook (``rb_set_profile_events``)
    records a second event pair around the dominant kernel of the step's last call
    that has one (the dense scan's full-corpus pass, or st::search's scorer)."""
    from retrieve_b200 import _lib

    lib = _lib.lib()
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for ka, kb in kev:  # a torch event gets its CUDA handle at its first record
        ka.record()
        kb.record()
    torch.cuda.synchronize()
    for (a, b), (ka, kb) in zip(evs, kev):
        if kernel:
            lib.rb_set_profile_events(ka.cuda_event, kb.cuda_event)
        a.record()
        step()
        b.record()
    lib.rb_set_profile_events(None, None)
    torch.cuda.synchronize()
    ts = [a.elapsed_time(b) for a, b in evs]
    kms = None
    if kernel:
        try:
            kms = statistics.mean(a.elapsed_time(b) for a, b in kev)
        except RuntimeError:  # the step made no call with a hooked kernel
            kms = None
    return statistics.mean(ts), kms


def _cpu(fn, sample_desc: str, scale: float, kind: str, cores: int | None = None) -> dict:
    """Times ``fn()`` once on the host (every core torch may use) → a cpu_baseline dict;
    ``scale`` turns one call into queries of the full workload (queries / fraction of the
    corpus covered)."""
    import os
    import time

    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.perf_counter()
    fn()
    dt = time.perf_counter() - t0
    return {"value": scale / dt, "unit": "queries/s", "cores": cores or os.cpu_count(), "kind": kind,
            "sample": f"{sample_desc} ({dt:.1f} s)"}


def _peaks() -> dict:
    pk = bench.ROOT / "MEASURED_PEAKS.json"
    return json.loads(pk.read_text()) if pk.exists() else {}


def _line(metric, value, unit, config, roofline, clocks, dtype, higher=True, **extra):
    d = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "higher_is_better": higher,
         "dtype": dtype, "data": "synthetic", "config": config, "roofline": roofline, "clocks": clocks}
    d.update(extra)
    print(json.dumps(d), flush=True)


# ---------------------------------------------------------------------------
# C4: int8
# ---------------------------------------------------------------------------
def run_c4(args, dev) -> dict:
    from retrieve_b200 import ops

    n = args.n_items if args.n_items != bench.N_ITEMS else 30_000_000
    d, b, k = 256, 4096, args.k
    cent = _centres(d, dev)
    codes = torch.empty((n, d), dtype=torch.int8, device=dev)
    scales = torch.empty((n,), dtype=torch.float32, device=dev)
    for lo, hi, x in _blocks(n, lambda r, sd: _mixture(cent, r, sd)):
        sc = x.abs().amax(dim=1).clamp_min(1e-8) / 127.0
        codes[lo:hi] = torch.round(x / sc[:, None]).clamp(-127, 127).to(torch.int8)
        scales[lo:hi] = sc
        del x
    q = _mixture(cent, b, 7)
    torch.cuda.synchronize()
    sampler = bench.ClockSampler(dev)
    sampler.start()
    ms, kms = _time(lambda: ops.int8_topk(q, codes, scales, k), args.warmup, args.steps)
    clocks = bench.ClockSampler.summary([(sampler.stop(), sampler.error)])
    peak = 2 * _peaks().get("bf16_tflops", 1590.0)
    ops_ = 2.0 * b * n * d
    achieved = ops_ / (kms / 1e3) / 1e12
    # CPU: the int32 scoring path restated in torch (int8 values in fp32 give exact int32
    # dots below 2^24), dequant (fp32(dot) * q_scale) * item_scale, top-k, on a sample
    qs_n, m = 4, min(n, 2_000_000)
    q_codes, q_scales = ops.quantize_int8(q[:qs_n])
    qc, qsc = q_codes.float().cpu(), q_scales.cpu()
    xc, xsc = codes[:m].float().cpu(), scales[:m].cpu()

    def cpu_step():
        sc_ = ((qc @ xc.t()) * qsc[:, None]) * xsc[None, :]
        return torch.topk(sc_, k, dim=1)

    cpu = _cpu(cpu_step, f"{qs_n} queries x the first {m} of {n} items (int32 dots as exact fp32 matmul, "
               "dequant, top-k; a restatement of the SilverTorch int32 path)", qs_n * m / n, "port")
    del codes, scales
    return {"metric": "queries/s @30M items d=256 int8 per-row scales, B=4096, k=100", "value": b / (ms / 1e3),
            "unit": "queries/s", "ms_per_step": ms, "higher_is_better": True, "dtype": "int8 -> int32",
            "config": {"workload": "int8 scoring (BASELINE config 4)", "n_items": n, "dim": d, "batch": b, "k": k,
                       "corpus": "1024-centre Gaussian mixture, sigma 0.15, per-row symmetric int8",
                       "step": "query quantization + int8 scan (tcgen05 kind::i8) + merge"},
            "roofline": {"bound": "tensor", "kernel": "dense_scan (int8, full-corpus pass)", "achieved": achieved,
                         "peak": peak, "unit": "TOP/s", "frac": achieved / peak, "kernel_ms": kms,
                         "peak_source": "derived: 2 x measured bf16 burst (the int8 tensor rate is twice bf16)"},
            "clocks": clocks, "cpu_baseline": cpu}


# ---------------------------------------------------------------------------
# C5: 1-bit pool + rerank
# ---------------------------------------------------------------------------
def _simhash(x: torch.Tensor, r: torch.Tensor) -> torch.Tensor:
    bits = (x.float() @ r.t() > 0).to(torch.int64)  # [n, 64 W]
    w = bits.shape[1] // 64
    shifts = torch.arange(64, device=x.device, dtype=torch.int64)
    return (bits.view(-1, w, 64) << shifts).sum(dim=2)  # disjoint bits: the sum is the OR


def run_c5(args, dev) -> dict:
    from retrieve_b200.bitknn import PackedBitsIndex, onebit_rerank_topk
    from retrieve_b200.quantize import project_simhash_1bit_query

    n = args.n_items if args.n_items != bench.N_ITEMS else 30_000_000
    d, nbits, b, pool, k = 128, 512, args.batch, 1000, args.k
    cent = _centres(d, dev)
    g = torch.Generator(device=dev).manual_seed(0)
    proj = torch.randn(nbits, d, generator=g, device=dev)
    items = torch.empty((n, d), dtype=torch.float16, device=dev)
    codes = torch.empty((n, nbits // 64), dtype=torch.int64, device=dev)
    for lo, hi, x in _blocks(n, lambda r, sd: _mixture(cent, r, sd)):
        items[lo:hi] = x.to(torch.float16)
        codes[lo:hi] = _simhash(x, proj)
        del x
    qf = _mixture(cent, b, 7)
    q = qf.to(torch.float16)
    m = min(n, 2_000_000)
    codes_host, items_host = codes[:m].cpu(), items[:m].cpu()
    index = PackedBitsIndex(codes)
    del codes
    torch.cuda.synchronize()

    def step():
        # the query side of SimHashKNN.forward (bit_knn.py:153-155): project, pack, search, rerank
        qbits = project_simhash_1bit_query(qf, proj)
        return onebit_rerank_topk(q, qbits, index, items, pool, k)

    sampler = bench.ClockSampler(dev)
    sampler.start()
    ms, kms = _time(step, args.warmup, args.steps)
    clocks = bench.ClockSampler.summary([(sampler.stop(), sampler.error)])
    peak = 2 * _peaks().get("bf16_tflops", 1590.0)
    ops_ = 2.0 * b * n * nbits  # the +-1 fp8 scan's multiply-adds
    achieved = ops_ / (kms / 1e3) / 1e12 if kms else None
    # CPU: the reference's own torch ops (popcount Hamming top-pool, then the gather + bmm
    # rerank), from its installed package, on a sample; else no CPU figure
    cpu = None
    ref_site = bench.REF_SITE
    if (ref_site / "retrieve").is_dir():
        import sys

        if str(ref_site) not in sys.path:
            sys.path.insert(0, str(ref_site))
        from retrieve.ops.reference.fused_masked_knn_topk import fused_masked_knn_topk as ref_rerank
        from retrieve.ops.reference.oporp_1bit_match_topk import oporp_1bit_match_topk_full as ref_hamming

        qs_n = 2
        qbits_host = project_simhash_1bit_query(qf[:qs_n], proj).cpu()
        q_host = q[:qs_n].cpu()

        def cpu_step():
            cand, _ = ref_hamming(qbits_host, codes_host, pool)
            cnt = torch.full((qs_n,), pool, dtype=torch.int64)
            return ref_rerank(q_host, items_host, cand, cnt, k)

        cpu = _cpu(cpu_step, f"{qs_n} queries x the first {m} of {n} items, the reference's torch ops "
                   "oporp_1bit_match_topk_full + fused_masked_knn_topk", qs_n * m / n, "reference")
    del index, items
    return {"metric": "queries/s @30M items 512-bit codes, pool 1000 + fp16 rerank d=128 to k=100, B=1024",
            "value": b / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms, "higher_is_better": True,
            "dtype": "fp8 (+-1) -> fp32 exact; fp16 rerank",
            "config": {"workload": "1-bit coarse retrieval + rerank (BASELINE config 5)", "n_items": n,
                       "bits": nbits, "batch": b, "pool": pool, "k": k,
                       "codes": "SimHash (N(0,1) projections, seed 0) of the mixture",
                       "stage1": "codes as a +-1 fp8 table, kind::f8f6f4 scan, exact 64W - 2*hamming scores",
                       "step": "query SimHash projection + sign packing, 1-bit pool, fp16 rerank"},
            "roofline": {"bound": "tensor", "kernel": "dense_scan (+-1 fp8, stage-1 pass)", "achieved": achieved,
                         "peak": peak, "unit": "TOP/s", "frac": achieved / peak if achieved else None,
                         "kernel_ms": kms,
                         "peak_source": "derived: 2 x measured bf16 burst (the fp8 tensor rate is twice bf16)"},
            "clocks": clocks, "cpu_baseline": cpu}


# ---------------------------------------------------------------------------
# C3: attribute-filtered
# ---------------------------------------------------------------------------
CARDS = (10, 20, 50, 100, 200, 500, 1000, 1000)


def _zipf_attrs(n: int, dev) -> torch.Tensor:
    g = torch.Generator(device=dev).manual_seed(5)
    cols = []
    for card in CARDS:
        p = 1.0 / torch.arange(1, card + 1, device=dev, dtype=torch.float64) ** 1.1
        cols.append(torch.multinomial((p / p.sum()).float(), n, replacement=True, generator=g))
    return torch.stack(cols, dim=1).to(torch.int64).view(n, len(CARDS), 1).contiguous()


def _predicates_for(attrs: torch.Tensor, b: int, target: float, seed: int) -> list[str]:
    """1-3 term expressions near the target selectivity: a term (c == v) whose
    frequency is within a factor of 1.5 of the target; for 50 %, OR of the most
    frequent values of a clause; for 1 %, some as the AND of two terms."""
    import random

    rnd = random.Random(seed)
    n = attrs.shape[0]
    freqs = [torch.bincount(attrs[:, c, 0], minlength=card).double().div(n).cpu().tolist()
             for c, card in enumerate(CARDS)]
    near = [(c, v) for c in range(len(CARDS)) for v, f in enumerate(freqs[c]) if target / 1.5 <= f <= target * 1.5]
    out = []
    for i in range(b):
        if target >= 0.5:
            c = rnd.randrange(3)
            order = sorted(range(CARDS[c]), key=lambda v: -freqs[c][v])
            acc, terms = 0.0, []
            for v in order:
                if acc >= target or len(terms) == 3:
                    break
                terms.append(f"{c}:{v}")
                acc += freqs[c][v]
            out.append(" OR ".join(terms))
        elif near and (target > 0.02 or i % 2 == 0):
            c, v = rnd.choice(near)
            out.append(f"{c}:{v}")
        else:  # AND of two independent ~sqrt(target) terms
            t = target ** 0.5
            pairs = [(c, v) for c in range(len(CARDS)) for v, f in enumerate(freqs[c]) if t / 1.5 <= f <= t * 1.5]
            (c1, v1), (c2, v2) = rnd.sample(pairs, 2) if len(pairs) > 1 else (pairs[0], pairs[0])
            out.append(f"{c1}:{v1} AND {c2}:{v2}")
    return out


def _expr_mask(a: torch.Tensor, e: str) -> torch.Tensor:
    """Items of ``a`` [M, C] (one value per clause) passing one expression of the forms
    ``_predicates_for`` writes: one term, an AND of two, an OR of up to three."""
    op = " OR " if " OR " in e else " AND "
    hits = [a[:, int(t.split(":")[0])] == int(t.split(":")[1]) for t in e.split(op)]
    m = hits[0]
    for h in hits[1:]:
        m = (m | h) if op == " OR " else (m & h)
    return m


def run_c3(args, dev) -> dict:
    from retrieve_b200 import ops
    from retrieve_b200.predicates import from_expressions

    n = args.n_items
    b, k = args.batch, args.k
    cent = bench.centres(dev)
    items = torch.empty((n, bench.DIM), dtype=torch.float16, device=dev)
    for lo, hi, x in _blocks(n, lambda r, sd: bench.mixture_block(cent, r, sd)):
        items[lo:hi] = x.to(torch.float16)
    q = bench.queries(cent, b).to(torch.float16)
    attrs = _zipf_attrs(n, dev)
    bloom = ops.bloom_build(attrs, 3)
    slices = ops.bloom_slices(bloom)  # index build time, like the Bloom words
    results = {}
    sampler = bench.ClockSampler(dev)
    sampler.start()
    for target in (0.01, 0.10, 0.50):
        exprs = _predicates_for(attrs, b, target, seed=int(target * 1000))
        preds = from_expressions(exprs).to(dev)
        sel = _selectivity(attrs, exprs)
        torch.cuda.synchronize()
        ms, kms = _time(lambda: ops.dense_topk_filtered(q, items, k, preds.terms, preds.n_terms, "bloom_recheck",
                                                        attrs, bloom, slices), args.warmup, args.steps)
        results[f"{int(target * 100)}%"] = {"queries_per_s": b / (ms / 1e3), "ms_per_step": ms, "kernel_ms": kms,
                                            "measured_selectivity": sel}
    clocks = bench.ClockSampler.summary([(sampler.stop(), sampler.error)])
    peak = _peaks().get("bf16_tflops", 1590.0)
    r10 = results["10%"]
    achieved = 2.0 * b * n * bench.DIM / (r10["kernel_ms"] / 1e3) / 1e12 if r10["kernel_ms"] else None
    # CPU: fp32 scores, the predicates restated as torch masks, masked top-k, on a sample
    qs_n, m = 4, min(n, 1_000_000)
    exprs10 = _predicates_for(attrs, b, 0.10, seed=100)[:qs_n]
    xh, ah, qh = items[:m].float().cpu(), attrs[:m, :, 0].cpu(), q[:qs_n].float().cpu()

    def cpu_step():
        sc = qh @ xh.t()
        mask = torch.stack([_expr_mask(ah, e) for e in exprs10])
        return torch.topk(sc.masked_fill(~mask, float("-inf")), k, dim=1)

    cpu = _cpu(cpu_step, f"{qs_n} queries (10 % selectivity) x the first {m} of {n} items: fp32 scores, "
               "predicate masks, top-k (a restatement)", qs_n * m / n, "port")
    del items, attrs, bloom, slices
    return {"metric": "queries/s @10M items d=128 fp16, 8 attrs + 64-bit bloom, B=1024, k=100 (10 % selectivity)",
            "value": r10["queries_per_s"], "unit": "queries/s", "ms_per_step": r10["ms_per_step"],
            "higher_is_better": True, "dtype": "fp16",
            "config": {"workload": "attribute-filtered kNN (BASELINE config 3)", "n_items": n, "dim": bench.DIM,
                       "batch": b, "k": k, "attrs": "8 categorical, cardinalities 10..1000, Zipf(1.1)",
                       "bloom": "64-bit, 3 hashes", "mode": "bloom test + exact recheck (exact results)",
                       "sweep": results},
            "roofline": {"bound": "tensor", "kernel": "dense_scan (fp16, filtered full-corpus pass)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak if achieved else None, "kernel_ms": r10["kernel_ms"],
                         "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops, burst)",
                         "note": "2*B*N*D dense flops at 10 % selectivity"},
            "clocks": clocks, "cpu_baseline": cpu}


def _selectivity(attrs, exprs: list[str], sample: int = 1 << 20) -> float:
    """Mean exact fraction of a strided item sample passing each query's expression."""
    idx = torch.linspace(0, attrs.shape[0] - 1, sample, device=attrs.device).long()
    a = attrs[idx, :, 0]
    return float(torch.stack([_expr_mask(a, e).float().mean() for e in exprs]).mean())


# ---------------------------------------------------------------------------
# ops: every other kernel at a representative size
# ---------------------------------------------------------------------------
def run_ops(args, dev):
    from retrieve_b200 import ops
    from retrieve_b200.shard import merge_topk

    hbm = _peaks().get("hbm_gbs", 6650.0)
    rows = []
    sampler = bench.ClockSampler(dev)
    sampler.start()

    def measure(name, fn, bytes_, note, ops_=None, unit=None):
        ms, _ = _time(fn, args.warmup, args.steps, kernel=False)
        r = {"op": name, "ms": ms, "algorithmic_bytes": bytes_, "GB_s": bytes_ / (ms / 1e3) / 1e9,
             "frac_of_hbm": bytes_ / (ms / 1e3) / 1e9 / hbm, "note": note}
        if ops_ is not None:
            r["rate"] = ops_ / (ms / 1e3)
            r["rate_unit"] = unit
        rows.append(r)

    n = 10_000_000
    g = torch.Generator(device=dev).manual_seed(3)
    attrs = _zipf_attrs(n, dev)
    rev = torch.zeros(8, dtype=torch.bool, device=dev)
    qa = torch.full((16, 8), -1, dtype=torch.int64, device=dev)
    qa[:, 0] = torch.arange(16, device=dev) % 10
    measure("clause_mask", lambda: ops.clause_mask(attrs, rev, qa), n * 8 * 8 + 16 * n,
            "attrs [10M,8,1] int64 read once per 8-query row block, [16, 10M] bool out")
    scores = torch.randn(16, n, generator=g, device=dev)
    measure("clause_mask_scores", lambda: ops.clause_mask_scores(scores, attrs, rev, qa), n * 64 + 16 * n * 8,
            "+ [16, 10M] fp32 scores in and out")
    measure("clause_compact", lambda: ops.clause_compact(attrs, rev, qa), n * 64 + 8 * int(16 * n * 0.2),
            "attrs + passing ids out (about 20 %)")
    items_t = torch.randn(128, n, generator=g, device=dev).to(torch.float16)
    q1 = torch.randn(1, 128, generator=g, device=dev).to(torch.float16)
    measure("gemv_scores", lambda: ops.gemv_scores(q1, items_t), 128 * n * 2 + 4 * n, "[1,128] x [128, 10M] fp16")
    del items_t, scores
    items = torch.randn(n, 128, generator=g, device=dev).to(torch.float16)
    qb = torch.randn(1024, 128, generator=g, device=dev).to(torch.float16)
    cand = torch.randint(0, n, (1024, 1000), generator=g, device=dev)
    cnt = torch.full((1024,), 1000, dtype=torch.int64, device=dev)
    measure("fused_masked_knn_topk", lambda: ops.fused_masked_knn_topk(qb, items, cand, cnt, 100),
            1024 * 1000 * (256 + 8), "B=1024, P=1000 random row gathers, D=128 fp16, k=100")
    bits = torch.randint(0, 256, (1_000_000, 64), generator=g, device=dev, dtype=torch.uint8).view(torch.int64)
    qbits = torch.randint(0, 256, (1024, 64), generator=g, device=dev, dtype=torch.uint8).view(torch.int64)
    measure("oporp_1bit_match_topk_full (popcount)", lambda: ops.oporp_1bit_match_topk_full(qbits, bits, 100),
            bits.numel() * 8, "B=1024 x 1M items x 512 bits, k=100: POPC-pipe bound",
            ops_=1024 * 1_000_000 * 16, unit="popc32/s")
    measure("bits_to_pm1", lambda: ops.bits_to_pm1(bits), bits.numel() * 8 * 9, "1M x 512 bits -> 1M x 512 int8")
    xq = torch.randn(4096, 256, generator=g, device=dev)
    measure("quantize_int8", lambda: ops.quantize_int8(xq), 4096 * 256 * 5 + 4096 * 4, "[4096, 256] fp32")
    measure("bloom_build", lambda: ops.bloom_build(attrs, 3), n * 64 + n * 8, "[10M, 8, 1] attrs -> [10M] words")
    pi = torch.randint(0, n, (8, 1024, 100), generator=g, device=dev)
    ps = torch.randn(8, 1024, 100, generator=g, device=dev)
    measure("merge_topk (8 shards)", lambda: merge_topk(pi, ps, 100), 8 * 1024 * 100 * 12,
            "[8, 1024, 100] per-shard lists -> [1024, 100]: latency-bound")
    clocks = bench.ClockSampler.summary([(sampler.stop(), sampler.error)])
    _line("per-kernel throughput (HBM-bound kernels as a fraction of the measured copy bandwidth)",
          statistics.mean(r["frac_of_hbm"] for r in rows if "rate" not in r and "latency" not in r["note"]),
          "mean frac of measured HBM", {"workload": "kernel sweep", "ops": rows},
          {"bound": "hbm", "peak": hbm, "unit": "GB/s", "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)"},
          clocks, "mixed")


# ---------------------------------------------------------------------------
# ivf: SilverTorch's IVF phase 1 + st::search
# ---------------------------------------------------------------------------
def _ivf_cpu_baseline(q, probe, offsets, sizes, codes_sorted, perm, gs, k, width, sample: int = 8) -> dict:
    """The reference's CPU path for phase 2 + 3 on ``sample`` queries, as the oracle's port
    (oracle/ivf.py: the reference scorer's int32 dots, top-k on the raw score, the
    two-multiply epilogue). The reference's own compiled CPU scorer cannot be loaded into
    this process: its library defines the st:: schemas that retrieve_b200.st has defined."""
    import time

    from oracle import ivf

    qs = q[:sample].cpu().numpy()
    pr = probe[:sample].cpu().numpy()
    args = (offsets.cpu().numpy(), sizes.cpu().numpy(), codes_sorted.cpu().numpy(), perm.cpu().numpy(),
            gs.cpu().numpy())
    t0 = time.perf_counter()
    ivf.search(qs, pr, args[0], args[1], args[2], args[3], args[4], k, width)
    dt = time.perf_counter() - t0
    return {"value": sample / dt, "unit": "queries/s", "cores": 1, "kind": "port",
            "sample": f"{sample} queries of the batch, phase 2 + 3 only (probe lists given)"}


def _ivf_inputs(args, dev):
    """The IVF workload's index and query batch (C2's mixture clustered by its nearest
    normalised centre, int8 codes with one global scale), built with this library's
    ``retrieve::`` ops only (no ``st`` schema), so that the reference arm can build the same
    inputs beside the reference's own ``st`` library."""
    from retrieve_b200 import ops
    from retrieve_b200.quantize import quantize_int8_global

    n = args.n_items
    d, b, k, n_probe = bench.DIM, args.batch, args.k, 16
    cent = bench.centres(dev)
    n_lists = cent.shape[0]
    items = torch.empty((n, d), dtype=torch.float32, device=dev)
    assign = torch.empty((n,), dtype=torch.int64, device=dev)
    centroids = (cent / cent.norm(dim=1, keepdim=True)).to(torch.bfloat16).contiguous()
    for lo, hi, x in _blocks(n, lambda r, sd: bench.mixture_block(cent, r, sd)):
        items[lo:hi] = x
        # build time: each item's list is its nearest centroid by dot product (phase 1's metric)
        assign[lo:hi] = (x.float() @ centroids.float().t()).argmax(dim=1)
    perm = torch.sort(assign, stable=True).indices  # sorted position -> item id
    sizes = torch.bincount(assign, minlength=n_lists)
    offsets = torch.zeros(n_lists + 1, dtype=torch.int64, device=dev)
    offsets[1:] = sizes.cumsum(0)
    codes_sorted, gs_f = quantize_int8_global(items, rows=perm)
    del items
    gs = torch.tensor(gs_f, dtype=torch.float32, device=dev)
    q = bench.queries(cent, b).to(torch.float32)
    qb = q.to(torch.bfloat16)
    probe0 = ops.dense_topk(qb, centroids, n_probe)[0]
    width = int(sizes[probe0].sum(1).max()) + 32 * n_probe  # room for other batches' probe totals
    torch.cuda.synchronize()
    return dict(n=n, d=d, b=b, k=k, n_probe=n_probe, n_lists=n_lists, centroids=centroids, perm=perm,
                sizes=sizes, offsets=offsets, codes_sorted=codes_sorted, gs=gs, q=q, qb=qb, probe0=probe0,
                width=width)


def _ids_digest(ids: torch.Tensor) -> str:
    import hashlib

    return hashlib.sha256(ids.to(torch.int64).cpu().numpy().tobytes()).hexdigest()[:16]


def run_ivf(args, dev):
    import retrieve_b200.st  # noqa: F401  (registers torch.ops.st.search)
    from retrieve_b200 import ops

    w = _ivf_inputs(args, dev)
    n, d, b, k, n_probe, n_lists = w["n"], w["d"], w["b"], w["k"], w["n_probe"], w["n_lists"]
    centroids, perm, sizes, offsets = w["centroids"], w["perm"], w["sizes"], w["offsets"]
    codes_sorted, gs, q, qb, probe0, width = w["codes_sorted"], w["gs"], w["q"], w["qb"], w["probe0"], w["width"]

    from retrieve_b200 import st

    def step():  # the registered op (it scores by cluster here: no bloom plans)
        probe = ops.dense_topk(qb, centroids, n_probe)[0]
        return torch.ops.st.search(q, probe, offsets, sizes, codes_sorted, perm, gs, k, width)

    def step_rows():
        probe = ops.dense_topk(qb, centroids, n_probe)[0]
        return st.search_rows(q, probe, offsets, sizes, codes_sorted, perm, gs, k, width)

    a, b_ = step(), step_rows()
    same = bool(torch.equal(a[0], b_[0]) and torch.equal(a[1], b_[1]))
    digest = _ids_digest(torch.ops.st.search(q, probe0, offsets, sizes, codes_sorted, perm, gs, k, width)[0])
    sampler = bench.ClockSampler(dev)
    sampler.start()
    ms, kms = _time(step, args.warmup, args.steps)
    ms_rows, kms_rows = _time(step_rows, args.warmup, args.steps)
    # st::search alone on phase 1's probes: the span `--impl reference --workload ivf` times
    # for the reference's own CUDA op
    ms_search, _ = _time(lambda: torch.ops.st.search(q, probe0, offsets, sizes, codes_sorted, perm, gs, k, width),
                         args.warmup, args.steps, kernel=False)
    bloom = _ivf_bloom_timing(args, dev, q, qb, centroids, n_probe, offsets, sizes, codes_sorted, perm, gs, k, width)
    clocks = bench.ClockSampler.summary([(sampler.stop(), sampler.error)])
    scored = float(sizes[probe0].sum())  # probed (query, item) pairs per batch
    hbm = _peaks().get("hbm_gbs", 6650.0)
    achieved = scored * d / (kms / 1e3) / 1e9 if kms else None
    cpu = _ivf_cpu_baseline(q, probe0, offsets, sizes, codes_sorted, perm, gs, k, width)
    del codes_sorted
    return {"metric": "queries/s, IVF phase 1 + st::search @10M items d=128 int8 (global scale), 1024 lists, "
                      "16 probes, B=1024, k=100", "value": b / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms,
            "higher_is_better": True, "dtype": "int8 -> int32",
            "config": {"workload": "SilverTorch IVF search (st::search semantics)", "n_items": n, "dim": d,
                       "batch": b, "k": k, "n_lists": n_lists, "n_probe": n_probe, "max_tensor_size_per_row": width,
                       "probed_pairs_per_batch": scored,
                       "scorer": "the registered op: scored by cluster, each probed cluster read once per group of "
                                 "up to 128 probing rows, tcgen05 kind::i8 MMA",
                       "rows": {"queries_per_s": b / (ms_rows / 1e3), "ms_per_step": ms_rows,
                                "kernel_ms": kms_rows, "identical_to_the_op": same},
                       "search_only": {"queries_per_s": b / (ms_search / 1e3), "ms_per_step": ms_search,
                                       "ids_sha256_16": digest,
                                       "note": "torch.ops.st.search alone on fixed probes (phase 2 + 3)"},
                       "bloom": bloom,
                       "corpus": "the C2 mixture, clustered by its nearest normalised centre, int8 with one global "
                                 "scale"},
            "roofline": {"bound": "hbm", "kernel": "st::search scorer", "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm if achieved else None, "kernel_ms": kms,
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)",
                         "note": "probed code bytes (pairs x D) per second of the scorer; rows probed by several "
                                 "queries of a batch are re-read from L2, so this can exceed the HBM copy rate"},
            "clocks": clocks, "cpu_baseline": cpu}


def _ivf_bloom_timing(args, dev, q, qb, centroids, n_probe, offsets, sizes, codes_sorted, perm, gs, k, width):
    """st::search under SilverTorch's bloom filter alone (no exact recheck), the study's timed
    setting: 3 attribute clauses per item (cardinalities 10, 20, 50, one value each), a 64-bit
    bloom with 3 positions per value (``bloom_index_build_fixed``), one single-term expression per
    query parsed by the library's parser. Row and grouped paths timed like the unfiltered ones; a
    failure here is reported in the config and leaves the headline line alone."""
    from retrieve_b200 import ops, st, st_bloom

    try:
        n, b = codes_sorted.shape[0], q.shape[0]
        g = torch.Generator(device=dev).manual_seed(7)
        card = torch.tensor([10, 20, 50], device=dev)
        vals = (torch.rand((n, 3), generator=g, device=dev) * card).to(torch.int64)  # sorted-position order
        fid = torch.arange(3, dtype=torch.int32, device=dev)
        foff = torch.arange(3 * n + 1, dtype=torch.int64, device=dev)
        index, boff = st.bloom_index_build_fixed(fid, foff, vals.reshape(-1), 64, 3)
        del vals, foff
        rng = torch.Generator().manual_seed(8)
        clause = torch.randint(0, 3, (b,), generator=rng)
        value = (torch.rand(b, generator=rng) * torch.tensor([10, 20, 50])[clause]).to(torch.int64)
        exprs = [f"{int(c)}:{int(v)}" for c, v in zip(clause, value)]
        _, (data, offs) = st_bloom.parse_expression_query_batch(exprs, torch.ones(b, dtype=torch.int64), 7)
        blob, slots, depth = st_bloom.prepare_plans(data, offs, dev)
        kw = dict(bloom_index=index, bloom_bundle_b_offsets=boff, plans=blob, plan_count=slots,
                  max_stack_size=depth, bloom_k=3, hash_k=7)

        def step_bloom():  # the registered op: bloom plans without the recheck score row by row
            probe = ops.dense_topk(qb, centroids, n_probe)[0]
            return torch.ops.st.search(q, probe, offsets, sizes, codes_sorted, perm, gs, k, width, **kw)

        def step_bloom_grouped():
            probe = ops.dense_topk(qb, centroids, n_probe)[0]
            return st.search_grouped(q, probe, offsets, sizes, codes_sorted, perm, gs, k, width, **kw)

        r1, r2 = step_bloom(), step_bloom_grouped()
        same = bool(torch.equal(r1[0], r2[0]) and torch.equal(r1[1], r2[1]))
        kept = float((r1[0] >= 0).float().mean())
        ms_b, _ = _time(step_bloom, args.warmup, args.steps, kernel=False)
        ms_bg, _ = _time(step_bloom_grouped, args.warmup, args.steps, kernel=False)
        return {"queries_per_s": b / (ms_b / 1e3), "step_ms": ms_b,
                "grouped_queries_per_s": b / (ms_bg / 1e3), "grouped_step_ms": ms_bg,
                "grouped_identical_to_row_path": same, "filled_result_fraction": kept,
                "filter": "one attribute term per query, 64-bit bloom, 3 positions, hash_k 7, no recheck"}
    except Exception as exc:  # noqa: BLE001  (a secondary measurement; the headline stands)
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


def measure_configs(args, dev, names=("c3", "c4", "c5", "ivf")) -> dict:
    """The other configurations' records, one after another on this GPU (each frees its
    inputs before the next); a failure is recorded in place of its record."""
    out = {}
    runners = {"c3": run_c3, "c4": run_c4, "c5": run_c5, "ivf": run_ivf}
    for name in names:
        try:
            out[name] = runners[name](args, dev)
        except Exception as exc:  # noqa: BLE001  (one config's failure leaves the others and the headline)
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


def reference_ivf(args, dev) -> dict:
    """The reference's own CUDA ``st::search`` (SilverTorch fork_search_cuda.cu, built from its
    sources by ``oracle/build_ref.py --cuda``) on the IVF workload's inputs, timed like this
    library's op: the same index and probes, ``torch.ops.st.search`` alone (phase 2 + 3)."""
    lib = Path(__file__).resolve().parent / "oracle" / "_ref" / "silvertorch_ref_cuda" / "silvertorch_ref_cuda.so"
    if not lib.exists():
        return {"impl": "reference", "unavailable": "the reference's CUDA ops were not built "
                "(python oracle/build_ref.py <checkout> --cuda)"}
    torch.ops.load_library(str(lib))
    w = _ivf_inputs(args, dev)
    b, k = w["b"], w["k"]
    call = (w["q"], w["probe0"], w["offsets"], w["sizes"], w["codes_sorted"], w["perm"], w["gs"], k, w["width"])
    out = torch.ops.st.search(*call)
    digest = _ids_digest(out[0])
    sampler = bench.ClockSampler(dev)
    sampler.start()
    ms, _ = _time(lambda: torch.ops.st.search(*call), args.warmup, args.steps, kernel=False)
    clocks = bench.ClockSampler.summary([(sampler.stop(), sampler.error)])
    value = b / (ms / 1e3)
    return {"metric": "queries/s, st::search alone (phase 2 + 3) @10M items d=128 int8 (global scale), 1024 "
                      "lists, 16 probes, B=1024, k=100", "value": value, "unit": "queries/s", "ms_per_step": ms,
            "higher_is_better": True, "impl": "reference", "dtype": "int8 -> int32",
            "config": {"workload": "SilverTorch IVF search (st::search), the reference's own CUDA op",
                       "n_items": w["n"], "batch": b, "k": k, "n_probe": w["n_probe"],
                       "max_tensor_size_per_row": w["width"], "ids_sha256_16": digest,
                       "library": "oracle/_ref/silvertorch_ref_cuda (the reference's *.cpp + *_cuda.cu, sm_100a)"},
            "clocks": clocks,
            "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_workload(args):
    import os

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--workload c3/c4/c5/ivf/ops runs on one GPU (no torchrun)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.workload == "ops":
        run_ops(args, dev)
        return
    if getattr(args, "impl", "ours") == "reference":
        if args.workload != "ivf":
            print(json.dumps({"impl": "reference", "unavailable": f"no reference arm for --workload {args.workload} "
                              "(its CPU baseline is part of the configuration's own line)"}), flush=True)
            return
        rec = reference_ivf(args, dev)
        line = {"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "data": "synthetic"}
        line.update(rec)
        print(json.dumps(line), flush=True)
        return
    rec = {"c3": run_c3, "c4": run_c4, "c5": run_c5, "ivf": run_ivf}[args.workload](args, dev)
    line = {"metric": rec.pop("metric"), "value": rec.pop("value"), "unit": rec.pop("unit"), "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "data": "synthetic"}
    line.update(rec)
    print(json.dumps(line), flush=True)
