"""Config 5 (1-bit candidates + exact rerank) and the kernel paths it needs:
512-byte rows (int8 D = 512, bf16 D = 256), k up to 1024 (dense scan and
popcount scan), the ±1 expansion of 1-bit codes, the tensor-core 1-bit top-k,
the LiNR V3 cascade, and its row-sharded two-exchange plan (shards run in
sequence on one GPU). All against the CPU oracle, bit for bit: Hamming scores
and int8 dots are integers, and the rerank's fp32 dots follow the oracle's
accumulation only up to rounding, so the rerank data is integer-valued."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import dense, knn
from oracle.bits import pack_signs
from tests.helpers import assert_topk_equal_up_to_ties, assert_topk_exact, make_int_rows, make_rows

pytestmark = pytest.mark.gpu


def _bits(n, w, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (n, 8 * w), generator=g, dtype=torch.uint8).view(torch.int64)


def _clustered_bits(n, w, seed, centres=64, flip=0.1):
    """Codes near a few centres (many near-ties, like SimHash codes of a mixture)."""
    g = torch.Generator().manual_seed(seed)
    c = torch.randn(centres, 64 * w, generator=g)
    x = c[torch.randint(0, centres, (n,), generator=g)] + flip * 4 * torch.randn(n, 64 * w, generator=g)
    return torch.from_numpy(pack_signs(x.numpy()))


def test_bits_to_pm1_matches_bit_order():
    from retrieve_b200 import ops

    bits = _bits(1000, 8, 1)
    pm1 = ops.bits_to_pm1(bits.cuda()).cpu()
    shifts = torch.arange(64)
    expect = ((bits[:, :, None] >> shifts) & 1).reshape(1000, 512) * 2 - 1
    assert torch.equal(pm1.to(torch.int64), expect)
    e4 = ops.bits_to_pm1(bits.cuda(), "e4m3").cpu()
    assert torch.equal(e4.view(torch.float8_e4m3fn).float().to(torch.int64), expect)


@pytest.mark.parametrize("w,b,n,k", [(8, 64, 100_000, 1000), (8, 300, 60_001, 100), (4, 200, 50_000, 256),
                                     (2, 130, 30_000, 37), (8, 96, 700, 1000)])
def test_tensor_core_onebit_topk_equals_popcount_oracle(w, b, n, k):
    from retrieve_b200.bitknn import PackedBitsIndex

    x = _clustered_bits(n, w, seed=w + n)
    q = _clustered_bits(b, w, seed=b + 7)
    idx = PackedBitsIndex(x.cuda())
    assert idx.tensor_cores
    ids, scores = idx.topk(q.cuda(), k)
    ref_i, ref_s = knn.oporp_full(q.numpy(), x.numpy(), min(k, n))
    if k > n:
        ref_i = np.concatenate([ref_i, np.full((b, k - n), -1)], axis=1)
        ref_s = np.concatenate([ref_s, np.full((b, k - n), -np.inf, dtype=np.float32)], axis=1)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i, ref_s)


def test_e4m3_pm1_scan_equals_popcount_oracle():
    """The same 1-bit top-k on the fp8 tensor cores (+-1 as e4m3)."""
    from retrieve_b200 import _lib, ops

    b, n, w, k = 200, 40_000, 8, 300
    x = _clustered_bits(n, w, seed=13)
    q = _clustered_bits(b, w, seed=14)
    ids, scores = ops.scaled_topk(ops.bits_to_pm1(q.cuda(), "e4m3"), None, ops.bits_to_pm1(x.cuda(), "e4m3"), None,
                                  k, _lib.RB_E4M3)
    ref_i, ref_s = knn.oporp_full(q.numpy(), x.numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i, ref_s)


def test_popcount_op_k1000_equals_oracle():
    from retrieve_b200 import ops

    b, n, w, k = 70, 80_000, 8, 1000
    x = _clustered_bits(n, w, seed=3)
    q = _clustered_bits(b, w, seed=4)
    ids, scores = ops.oporp_1bit_match_topk_full(q.cuda(), x.cuda(), k)
    ref_i, ref_s = knn.oporp_full(q.numpy(), x.numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i, ref_s)


@pytest.mark.parametrize("b,n,k", [(64, 30_000, 100), (300, 20_003, 1000), (1024, 50_000, 500)])
def test_int8_d512_bit_exact(b, n, k):
    from retrieve_b200 import ops

    g = torch.Generator().manual_seed(n)
    xc = torch.randint(-128, 128, (n, 512), generator=g, dtype=torch.int64).to(torch.int8)
    qc = torch.randint(-128, 128, (b, 512), generator=g, dtype=torch.int64).to(torch.int8)
    xs = torch.rand(n, generator=g) + 0.5
    qs = torch.rand(b, generator=g) + 0.5
    ids, scores = ops.int8_codes_topk(qc.cuda(), qs.cuda(), xc.cuda(), xs.cuda(), k)
    # oracle: exact int64 dots, dequant (fp32(dot) * q_scale) * item_scale
    dots = qc.numpy().astype(np.int64) @ xc.numpy().astype(np.int64).T
    s = (dots.astype(np.float32) * qs.numpy()[:, None]).astype(np.float32) * xs.numpy()[None, :]
    from oracle.select import topk_strict

    ref_i, ref_s = topk_strict(s.astype(np.float32), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i, ref_s)


@pytest.mark.parametrize("b,n,d,k", [(300, 40_000, 256, 100), (64, 30_000, 128, 1000), (1024, 100_000, 128, 700),
                                     (200, 25_000, 256, 1024)])
def test_dense_wide_rows_and_large_k_exact(b, n, d, k):
    from retrieve_b200 import ops

    q = make_int_rows(b, d, seed=b, device="cuda")
    x = make_int_rows(n, d, seed=n, device="cuda")
    ids, scores = ops.dense_topk(q, x, k)
    ref_i, ref_s = dense.dense_topk(q.float().cpu().numpy(), x.float().cpu().numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i, ref_s)


def _c5_data(n, b, w=8, d=128, seed=0, integer=True):
    x_bits = _clustered_bits(n, w, seed=seed)
    q_bits = _clustered_bits(b, w, seed=seed + 1)
    if integer:
        x = make_int_rows(n, d, seed=seed + 2, dtype=torch.float16)
        q = make_int_rows(b, d, seed=seed + 3, dtype=torch.float16)
    else:
        x = make_rows(n, d, seed=seed + 2, dtype=torch.float16)
        q = make_rows(b, d, seed=seed + 3, dtype=torch.float16)
    return x_bits, q_bits, x, q


def test_onebit_rerank_cascade_equals_oracle():
    from retrieve_b200.bitknn import PackedBitsIndex, onebit_rerank_topk

    n, b, pool, k = 120_000, 128, 1000, 100
    x_bits, q_bits, x, q = _c5_data(n, b)
    idx = PackedBitsIndex(x_bits.cuda())
    ids, scores = onebit_rerank_topk(q.cuda(), q_bits.cuda(), idx, x.cuda(), pool, k)
    cand, _ = knn.oporp_full(q_bits.numpy(), x_bits.numpy(), pool)
    counts = (cand >= 0).sum(axis=1)
    ref_i, ref_s = knn.fused_masked_knn_topk(q.float().numpy(), x.float().numpy(), cand, counts, k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i, ref_s)


@pytest.mark.parametrize("world", [2, 8])
def test_sharded_cascade_equals_single_gpu(world):
    """The two-exchange plan, every rank's calls in sequence on one GPU; the
    all-gather + merge is emulated by stacking + merge_topk. The pool is the
    single-GPU pool exactly; in the rerank, equal fp32 scores of different items
    are ordered by global id across shards but by pool position on one GPU, so
    ids may differ inside runs of equal scores (the scores may not)."""
    from retrieve_b200.bitknn import PackedBitsIndex, onebit_rerank_topk
    from retrieve_b200.shard import merge_topk, shard_bounds
    from retrieve_b200 import ops

    n, b, pool, k = 200_003, 256, 1000, 100
    x_bits, q_bits, x, q = _c5_data(n, b, seed=10, integer=False)
    xb, qb, xe, qe = x_bits.cuda(), q_bits.cuda(), x.cuda(), q.cuda()
    ref_i, ref_s = onebit_rerank_topk(qe, qb, PackedBitsIndex(xb), xe, pool, k)
    bounds = [shard_bounds(n, world, r) for r in range(world)]
    st1 = [PackedBitsIndex(xb[lo:hi].contiguous()).topk(qb, pool, lo) for lo, hi in bounds]
    pool_ids, _ = merge_topk(torch.stack([a for a, _ in st1]), torch.stack([s for _, s in st1]), pool)
    st2 = []
    for lo, hi in bounds:
        local = pool_ids - lo
        counts = torch.full((b,), pool, dtype=torch.int64, device="cuda")
        i2, s2 = ops.fused_masked_knn_topk(qe, xe[lo:hi].contiguous(), local, counts, k)
        st2.append((torch.where(i2 >= 0, i2 + lo, i2), s2))
    ids, scores = merge_topk(torch.stack([a for a, _ in st2]), torch.stack([s for _, s in st2]), k)
    torch.cuda.synchronize()
    assert_topk_equal_up_to_ties(ids.cpu().numpy(), scores.cpu().numpy(), ref_i.cpu().numpy(), ref_s.cpu().numpy())
