"""Int8 scoring + top-k against the CPU oracle: int32 dots
are exact, the dequant order is the reference's, so ids and scores are
bit-exact, ties toward the lower id."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import knn
from tests.helpers import assert_topk_exact

pytestmark = pytest.mark.gpu


def _items(n, d, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g)
    scales = x.abs().amax(dim=1).clamp_min(1e-8) / 127.0
    codes = torch.round(x / scales[:, None]).clamp(-127, 127).to(torch.int8)
    return codes, scales.to(torch.float32)


@pytest.mark.parametrize("b,n,d,k", [(64, 20_000, 256, 100), (300, 50_000, 256, 50), (130, 7_777, 128, 100),
                                     (1024, 300_000, 256, 100)])
def test_int8_topk_bit_exact(b, n, d, k):
    from retrieve_b200 import ops

    codes, scales = _items(n, d, seed=n)
    q = torch.randn(b, d, generator=torch.Generator().manual_seed(b))
    ids, scores = ops.int8_topk(q.cuda(), codes.cuda(), scales.cuda(), k)
    ref_ids, ref_scores = knn.int8_topk(q.numpy(), codes.numpy(), scales.numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


@pytest.mark.parametrize("short_rows", [1, 150])
def test_int8_speculative_seed_second_pass(short_rows):
    """The int8 full pass starts from a speculative seed (a high sampled chunk max). The first
    `short_rows` queries see their best items only in the sampled tiles (one per 32-item
    chunk, every 16th tile), so fewer than k items reach that seed: those rows come back
    short and run again from the safe seed, the first 128 as one compact batch, the rest
    with their query groups. The other rows are random. Bit for bit the oracle's."""
    from retrieve_b200 import ops

    b, n, d, k = 200, 400_000, 128, 10
    g = torch.Generator().manual_seed(43)
    codes = torch.randint(-3, 4, (n, d), generator=g).to(torch.int8)
    scales = torch.ones(n, dtype=torch.float32)
    q = torch.randn(b, d, generator=g)
    q[:short_rows] = 0
    q[:short_rows, 0], q[:short_rows, 1] = 16.0, 1.0  # quantized to codes 127 and 8
    tiles = torch.arange(0, n // 128, 16)
    heads = (tiles[:, None] * 128 + torch.arange(0, 128, 32)[None, :]).reshape(-1)
    r = torch.arange(heads.numel())
    codes[heads, 0] = (20 + r // 16).to(torch.int8)  # dots 127 x0 + 8 x1, distinct and rising with r
    codes[heads, 1] = (r % 16).to(torch.int8)
    ids, scores = ops.int8_topk(q.cuda(), codes.cuda(), scales.cuda(), k)
    ref_ids, ref_scores = knn.int8_topk(q.numpy(), codes.numpy(), scales.numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)
    assert set(ref_ids[0].tolist()) <= set(heads.tolist())


def test_int8_global_scale_equals_silvertorch_full_probe():
    """With one global item scale the ranking is the raw int32 dot's, as in
    SilverTorch's st::search with every cluster probed."""
    from retrieve_b200 import ops

    b, n, d, k = 96, 30_000, 256, 100
    g = torch.Generator().manual_seed(9)
    x = torch.randn(n, d, generator=g)
    gscale = float(x.abs().max() / 127.0)
    codes = torch.round(x / gscale).clamp(-127, 127).to(torch.int8)
    q = torch.randn(b, d, generator=g)
    ids, scores = ops.int8_topk(q.cuda(), codes.cuda(), torch.full((n,), gscale).cuda(), k)
    ref_ids, ref_scores = knn.silvertorch_fullprobe(q.numpy(), codes.numpy(), gscale, k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


@pytest.mark.parametrize("d", [128, 256])
def test_int8_tensor_core_dots_equal_reference_fused_kmean_ann(d):
    """Unit scales: every returned score is the raw int32 dot as fp32, which must
    equal SilverTorch's own CPU scorer's dot for that (query, item)
    (tests/golden/make_golden_int8.py), and the ids are its top-k with ties to
    the lower id."""
    import ctypes
    from pathlib import Path

    from oracle.select import topk_strict
    from retrieve_b200 import _lib

    g = np.load(Path(__file__).resolve().parent / "golden" / "golden_int8.npz")
    qc, xc, dots = g[f"queries_{d}"], g[f"items_{d}"], g[f"dots_{d}"]
    b, n, k = qc.shape[0], xc.shape[0], 100
    q = torch.from_numpy(qc).cuda()
    x = torch.from_numpy(xc).cuda()
    qs = torch.ones(b, dtype=torch.float32, device="cuda")
    xs = torch.ones(n, dtype=torch.float32, device="cuda")
    ids = torch.empty(b, k, dtype=torch.int64, device="cuda")
    scores = torch.empty(b, k, dtype=torch.float32, device="cuda")
    lib = _lib.lib()
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_workspace_size(b, n, d, _lib.RB_I8, k, ctypes.byref(nb)), "ws")
    ws = torch.empty(max(nb.value, 256), dtype=torch.uint8, device="cuda")
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.rb_dense_topk_i8(vp(q), vp(qs), vp(x), vp(xs), b, n, d, k, 0, vp(ids), vp(scores), vp(ws), ws.numel(),
                              stream)
    _lib.check(rc, "dense_topk_i8")
    torch.cuda.synchronize()
    ref_ids, ref_scores = topk_strict(dots.astype(np.float32), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)
