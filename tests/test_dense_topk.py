"""Parity of ``retrieve::dense_topk`` (fused tcgen05 scoring + exact top-k)
against the CPU oracle (oracle/dense.py, the reference's FullScanKNN /
PostfilterKNN semantics with ties to the lower id).

Integer-valued inputs make every fp32 dot exact whatever the accumulation order,
so those cases are bit-exact (scores and ids slot by slot, the strict tie rule
included). Real-valued inputs are gated at |score| error <= 1e-5 absolute and
recall@k >= 0.999 (the BASELINE tolerance is 1e-2 relative)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.dense import dense_topk as oracle_dense_topk
from tests.helpers import assert_topk_close, assert_topk_exact, make_int_rows, make_rows, mixture_rows

pytestmark = pytest.mark.gpu


def _run(q, x, k):
    from retrieve_b200 import ops

    ids, scores = ops.dense_topk(q.cuda(), x.cuda(), k)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), scores.cpu().numpy()


@pytest.mark.parametrize(
    "b,n,d,k",
    [
        (64, 5000, 128, 100),
        (1, 777, 128, 10),
        (130, 4099, 128, 100),  # ragged B (two query groups, second partial) and N
        (300, 20000, 64, 32),
        (128, 50, 128, 100),  # k > N: -1 / -inf tail
        (256, 100_000, 128, 1),
        (512, 30_000, 128, 256),
    ],
)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_dense_topk_integer_exact(b, n, d, k, dtype):
    q = make_int_rows(b, d, seed=11, dtype=dtype)
    x = make_int_rows(n, d, seed=12, dtype=dtype)
    ids, scores = _run(q, x, k)
    ref_ids, ref_scores = oracle_dense_topk(q, x, k)
    assert_topk_exact(ids, scores, ref_ids, ref_scores)


def test_dense_topk_sampled_levels_exact():
    """Large enough for the sampled threshold passes (level strides > 1)."""
    b, n, d, k = 256, 1_600_000, 128, 100
    q = make_int_rows(b, d, seed=21, lo=-2, hi=3)
    x = make_int_rows(n, d, seed=22, lo=-2, hi=3)
    ids, scores = _run(q, x, k)
    ref_ids, ref_scores = oracle_dense_topk(q, x, k)
    assert_topk_exact(ids, scores, ref_ids, ref_scores)


def _device_topk_ties_low(q, x, k, chunk=1 << 18):
    """Plain PyTorch reference on the GPU for integer-valued rows: fp32 matmul (exact here),
    then top-k on the 64-bit key (score << 32 | ~id), so ties go to the lower id."""
    best = None
    for lo in range(0, x.shape[0], chunk):
        s = (q.float() @ x[lo : lo + chunk].float().t()).to(torch.int64)
        ids = torch.arange(lo, lo + s.shape[1], device=q.device, dtype=torch.int64)
        key = (s << 32) | (0xFFFFFFFF - ids)[None, :]
        if best is not None:
            key = torch.cat([best, key], dim=1)
        best = torch.topk(key, min(k, key.shape[1]), dim=1).values
    ids = 0xFFFFFFFF - (best & 0xFFFFFFFF)
    return ids, (best >> 32).to(torch.float32)


def test_dense_topk_10m_integer_exact_on_device():
    """At the benchmark's shape (10M x 128 bf16, B = 1024, k = 100) the sampling pass's chunk
    maxima fill more workspace than the candidate lists; the seeds and counts sit past both.
    Checked against the PyTorch reference on the device (integer values: exact)."""
    from retrieve_b200 import ops

    b, n, d, k = 1024, 10_000_000, 128, 100
    g = torch.Generator(device="cuda").manual_seed(51)
    q = torch.randint(-8, 9, (b, d), generator=g, device="cuda").to(torch.bfloat16)
    x = torch.randint(-8, 9, (n, d), generator=g, device="cuda").to(torch.bfloat16)
    ids, scores = ops.dense_topk(q, x, k)
    ref_ids, ref_scores = _device_topk_ties_low(q, x, k)
    assert torch.equal(scores, ref_scores)
    assert torch.equal(ids, ref_ids)


def test_dense_topk_ascending_scores_compaction_storm():
    """Items ordered so every query's scores rise with the id: every item beats
    the running threshold, forcing list compaction on every chunk."""
    b, n, d, k = 64, 40_000, 128, 100
    q = torch.zeros(b, d)
    q[:, 0] = 1.0
    x = torch.zeros(n, d)
    x[:, 0] = (torch.arange(n) // 3).float()  # runs of 3 equal scores
    q, x = q.to(torch.bfloat16), x.to(torch.bfloat16)
    ids, scores = _run(q, x, k)
    ref_ids, ref_scores = oracle_dense_topk(q, x, k)
    assert_topk_exact(ids, scores, ref_ids, ref_scores)


@pytest.mark.parametrize("b", [64, 200, 512])
def test_dense_topk_compaction_storm_all_kernels(b):
    """Rising scores for every query (1-SM kernel at B <= 128, the CTA-pair
    kernel with one and two query groups above)."""
    n, d, k = 30_000, 128, 100
    g = torch.Generator().manual_seed(b)
    q = torch.zeros(b, d)
    q[:, 0] = 1.0
    q[:, 1] = torch.randint(0, 3, (b,), generator=g).float()
    x = torch.zeros(n, d)
    x[:, 0] = (torch.arange(n) // 5).float()
    x[:, 1] = torch.randint(0, 4, (n,), generator=g).float()
    q, x = q.to(torch.bfloat16), x.to(torch.bfloat16)
    ids, scores = _run(q, x, k)
    ref_ids, ref_scores = oracle_dense_topk(q, x, k)
    assert_topk_exact(ids, scores, ref_ids, ref_scores)


def test_dense_topk_all_ties_lowest_ids_win():
    b, n, d, k = 200, 9000, 128, 50
    q = torch.ones(b, d, dtype=torch.bfloat16)
    x = torch.ones(n, d, dtype=torch.bfloat16)
    ids, scores = _run(q, x, k)
    assert (scores == 128.0).all()
    assert (ids == np.arange(k)[None, :]).all()


def test_dense_topk_real_valued_close():
    b, n, d, k = 200, 60_000, 128, 100
    q = make_rows(b, d, seed=31, dtype=torch.bfloat16)
    x, centres = mixture_rows(n, d, n_centres=64, sigma=0.15, seed=32, dtype=torch.bfloat16)
    ids, scores = _run(q, x, k)
    ref_ids, ref_scores = oracle_dense_topk(q, x, k)
    assert_topk_close(ids, scores, ref_ids, ref_scores, rtol=0.0, atol=1e-5, min_recall=0.999)


def test_dense_topk_no_device_error_and_stream_order():
    """Runs on a side stream; outputs are complete once that stream is synced,
    and the kernel's device error word stays 0."""
    import ctypes

    from retrieve_b200 import _lib, ops

    b, n, d, k = 96, 10_000, 128, 20
    q = make_int_rows(b, d, seed=41).cuda()
    x = make_int_rows(n, d, seed=42).cuda()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ids, scores = ops.dense_topk(q, x, k)
    s.synchronize()
    ref_ids, ref_scores = oracle_dense_topk(q, x, k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)
    # direct C-ABI call to read the error word of the workspace it used
    lib = _lib.lib()
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_workspace_size(b, n, d, _lib.RB_BF16, k, ctypes.byref(nb)), "ws")
    ws = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
    out_i = torch.empty(b, k, dtype=torch.int64, device="cuda")
    out_s = torch.empty(b, k, dtype=torch.float32, device="cuda")
    rc = lib.rb_dense_topk(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(x.data_ptr()), b, n, d, _lib.RB_BF16, k, 5,
        ctypes.c_void_p(out_i.data_ptr()), ctypes.c_void_p(out_s.data_ptr()),
        ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
    )
    _lib.check(rc, "dense_topk")
    err = ctypes.c_int(-1)
    _lib.check(lib.rb_workspace_device_error(ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.byref(err)), "err")
    assert err.value == 0
    assert (out_i.cpu().numpy() == ref_ids + 5).all()  # id_offset shifts every id


def test_dense_topk_rejects_cpu_and_bad_shapes():
    from retrieve_b200 import ops

    x = torch.zeros(10, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        ops.dense_topk(torch.zeros(2, 64, device="cuda"), x, 5)
    with pytest.raises(TypeError):
        ops.dense_topk(torch.zeros(2, 128, device="cuda"), x.float(), 5)
    with pytest.raises(ValueError):
        ops.dense_topk(torch.zeros(2, 128, device="cuda"), x.t().contiguous().t(), 5)
