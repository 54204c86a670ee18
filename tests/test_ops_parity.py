"""GPU parity of the retrieve:: ops (retrieve_b200.ops) against the CPU oracle.
Integer paths (clause filter, compaction, Hamming, int8 quantization, and dots
of small-integer vectors) are bit-exact with ties broken toward the lower index;
real-valued dots are gated at 1e-5 absolute."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import filters, knn
from tests.golden import golden_inputs as gi
from tests.helpers import assert_topk_exact

pytestmark = pytest.mark.gpu


def _ops():
    from retrieve_b200 import ops

    return ops


def _attrs(n, c, a, b, seed, vocab=8, pad=0.3, inactive=0.2):
    g = torch.Generator().manual_seed(seed)
    attrs = torch.randint(0, vocab, (n, c, a), generator=g)
    attrs[torch.rand(n, c, a, generator=g) < pad] = -1
    q = torch.randint(0, vocab, (b, c), generator=g)
    q[torch.rand(b, c, generator=g) < inactive] = -1
    rev = torch.rand(c, generator=g) < 0.3
    return attrs, rev, q


@pytest.mark.parametrize("n,c,a,b", [(2000, 3, 4, 16), (1, 1, 1, 1), (5003, 8, 2, 33), (70_000, 2, 3, 4)])
def test_clause_mask_and_scores(n, c, a, b):
    ops = _ops()
    attrs, rev, q = _attrs(n, c, a, b, seed=n)
    m = ops.clause_mask(attrs.cuda(), rev.cuda(), q.cuda()).cpu().numpy()
    assert np.array_equal(m, filters.clause_mask(attrs.numpy(), rev.numpy(), q.numpy()))
    sc = torch.randn(b, n, generator=torch.Generator().manual_seed(1))
    out = ops.clause_mask_scores(sc.cuda(), attrs.cuda(), rev.cuda(), q.cuda()).cpu().numpy()
    assert np.array_equal(out, filters.clause_mask_scores(sc.numpy(), attrs.numpy(), rev.numpy(), q.numpy()))


def test_clause_ops_on_golden_inputs():
    ops = _ops()
    attrs, rev, q = gi.clause_inputs()
    ids, counts = ops.clause_compact(attrs.cuda(), rev.cuda(), q.cuda())
    ref_ids, ref_counts = filters.clause_compact(attrs.numpy(), rev.numpy(), q.numpy())
    counts = counts.cpu().numpy()
    assert np.array_equal(counts, ref_counts)
    ids = ids.cpu().numpy()
    for r in range(q.shape[0]):
        assert np.array_equal(ids[r, : counts[r]], ref_ids[r, : counts[r]])


@pytest.mark.parametrize("n,b", [(3000, 5), (1024 * 7 + 3, 2), (200_000, 3), (1, 1)])
def test_clause_compact_ascending_and_exact(n, b):
    ops = _ops()
    attrs, rev, q = _attrs(n, 3, 2, b, seed=b, vocab=4)
    ids, counts = ops.clause_compact(attrs.cuda(), rev.cuda(), q.cuda())
    ref_ids, ref_counts = filters.clause_compact(attrs.numpy(), rev.numpy(), q.numpy())
    counts = counts.cpu().numpy()
    ids = ids.cpu().numpy()
    assert np.array_equal(counts, ref_counts)
    for r in range(b):
        assert np.array_equal(ids[r, : counts[r]], ref_ids[r, : counts[r]])


def test_clause_compact_empty_corpus():
    ops = _ops()
    ids, counts = ops.clause_compact(torch.zeros(0, 2, 2, dtype=torch.int64, device="cuda"),
                                     torch.zeros(2, dtype=torch.bool, device="cuda"),
                                     torch.zeros(3, 2, dtype=torch.int64, device="cuda"))
    assert ids.shape == (3, 0) and counts.cpu().tolist() == [0, 0, 0]


@pytest.mark.parametrize("d,n", [(128, 4096), (64, 1000), (256, 777), (100, 16)])
def test_gemv_scores_bit_exact(d, n):
    ops = _ops()
    g = torch.Generator().manual_seed(d + n)
    q = torch.randn(1, d, generator=g).to(torch.float16)
    et = torch.randn(d, n, generator=g).to(torch.float16)
    out = ops.gemv_scores(q.cuda(), et.cuda()).cpu().numpy()
    assert np.array_equal(out, knn.gemv_scores(q.numpy(), et.numpy()))


def test_gemv_scores_rejects_bad_input():
    ops = _ops()
    with pytest.raises(ValueError):
        ops.gemv_scores(torch.zeros(2, 8, dtype=torch.float16, device="cuda"),
                        torch.zeros(8, 4, dtype=torch.float16, device="cuda"))


def _int_f16(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-3, 4, shape, generator=g).to(torch.float16)


@pytest.mark.parametrize("b,n,d,p,k", [(8, 3000, 64, 500, 20), (3, 50_000, 128, 40_000, 100), (5, 100, 32, 60, 60)])
def test_fused_masked_knn_topk_integer_exact(b, n, d, p, k):
    ops = _ops()
    g = torch.Generator().manual_seed(p)
    q, x = _int_f16((b, d), 1), _int_f16((n, d), 2)
    pos = torch.stack([torch.randperm(n, generator=g)[:p] for _ in range(b)])
    counts = torch.randint(0, p + 1, (b,), generator=g)
    counts[0] = p
    counts[-1] = 0
    ids, scores = ops.fused_masked_knn_topk(q.cuda(), x.cuda(), pos.cuda(), counts.cuda(), k)
    ref_ids, ref_scores = knn.fused_masked_knn_topk(q, x, pos, counts, k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


def test_fused_masked_knn_topk_golden_inputs_close():
    ops = _ops()
    q, x, pos, counts = gi.fmkt_inputs()
    ids, scores = ops.fused_masked_knn_topk(q.cuda(), x.cuda(), pos.cuda(), counts.cuda(), 20)
    ref_ids, ref_scores = knn.fused_masked_knn_topk(q, x, pos, counts, 20)
    np.testing.assert_allclose(scores.cpu().numpy(), ref_scores, atol=1e-5, rtol=0)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)


def test_fused_masked_knn_topk_mixed_dtypes_and_errors():
    ops = _ops()
    q, x = _int_f16((4, 64), 3), _int_f16((1000, 64), 4)
    pos = torch.arange(1000).repeat(4, 1)
    counts = torch.full((4,), 1000)
    ref = knn.fused_masked_knn_topk(q, x, pos, counts, 10)
    for qq, xx in [(q.float(), x), (q, x.float()), (q.float(), x.float())]:
        ids, scores = ops.fused_masked_knn_topk(qq.cuda(), xx.cuda(), pos.cuda(), counts.cuda(), 10)
        assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), *ref)
    with pytest.raises(ValueError):
        ops.fused_masked_knn_topk(q.cuda(), x.cuda(), pos[:, :5].contiguous().cuda(), counts.cuda(), 10)
    with pytest.raises(TypeError):
        ops.fused_masked_knn_topk(q.to(torch.bfloat16).cuda(), x.cuda(), pos.cuda(), counts.cuda(), 10)


@pytest.mark.parametrize("b,n,w,k", [(8, 5000, 2, 50), (130, 40_000, 8, 100), (3, 300, 4, 300), (64, 100_000, 8, 1)])
def test_oporp_full_exact(b, n, w, k):
    ops = _ops()
    g = torch.Generator().manual_seed(n)
    qb = torch.randint(-(2**63), 2**63 - 1, (b, w), generator=g, dtype=torch.int64)
    xb = torch.randint(-(2**63), 2**63 - 1, (n, w), generator=g, dtype=torch.int64)
    ids, scores = ops.oporp_1bit_match_topk_full(qb.cuda(), xb.cuda(), k)
    ref_ids, ref_scores = knn.oporp_full(qb.numpy(), xb.numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


@pytest.mark.parametrize("b,n,w,k", [(4, 20_000, 2, 3000), (3, 9000, 3, 100), (2, 5000, 1, 5000), (5, 70_000, 8, 1500)])
def test_oporp_full_counting_select_exact(b, n, w, k):
    """k past the list kernel (or an odd word count): the counting select, bit for bit the
    oracle with ties to the lower row (w = 1 leaves 65 distinct scores: ties at every rank)."""
    ops = _ops()
    g = torch.Generator().manual_seed(n + w)
    qb = torch.randint(-(2**63), 2**63 - 1, (b, w), generator=g, dtype=torch.int64)
    xb = torch.randint(-(2**63), 2**63 - 1, (n, w), generator=g, dtype=torch.int64)
    ids, scores = ops.oporp_1bit_match_topk_full(qb.cuda(), xb.cuda(), k)
    ref_ids, ref_scores = knn.oporp_full(qb.numpy(), xb.numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


def test_oporp_indirect_counting_select_exact():
    """min(k, P) past 224 (LiNR V3's candidate pools, 5000 by default): the counting select over
    each row's candidate slots, ragged counts included, bit for bit the oracle."""
    ops = _ops()
    g = torch.Generator().manual_seed(77)
    b, n, w, p, k = 6, 30_000, 2, 3000, 2000
    qb = torch.randint(-(2**63), 2**63 - 1, (b, w), generator=g, dtype=torch.int64)
    xb = torch.randint(-(2**63), 2**63 - 1, (n, w), generator=g, dtype=torch.int64)
    pos = torch.stack([torch.randperm(n, generator=g)[:p] for _ in range(b)])
    counts = torch.tensor([3000, 2500, 2000, 1999, 10, 0])
    ids, scores = ops.oporp_1bit_match_topk_indirect(qb.cuda(), xb.cuda(), k, pos.cuda(), counts.cuda())
    ref_ids, ref_scores = knn.oporp_indirect(qb.numpy(), xb.numpy(), k, pos.numpy(), counts.numpy())
    assert ids.shape == (b, k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


def test_oporp_indirect_exact_golden_inputs():
    ops = _ops()
    qb, xb, pos, counts = gi.oporp_inputs()
    ids, scores = ops.oporp_1bit_match_topk_indirect(qb.cuda(), xb.cuda(), 50, pos.cuda(), counts.cuda())
    ref_ids, ref_scores = knn.oporp_indirect(qb.numpy(), xb.numpy(), 50, pos.numpy(), counts.numpy())
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


def test_oporp_indirect_min_k_p_columns():
    ops = _ops()
    qb, xb, pos, counts = gi.oporp_inputs()
    ids, scores = ops.oporp_1bit_match_topk_indirect(qb.cuda(), xb.cuda(), 500, pos[:, :40].contiguous().cuda(),
                                                     counts.clamp_max(40).cuda())
    assert ids.shape == (8, 40)
    ref_ids, ref_scores = knn.oporp_indirect(qb.numpy(), xb.numpy(), 500, pos[:, :40].numpy(),
                                             counts.clamp_max(40).numpy())
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


def test_quantize_int8_bit_exact():
    ops = _ops()
    g = torch.Generator().manual_seed(9)
    for x in (gi.quantize_inputs(), torch.randn(10_000, 192, generator=g)):
        x = x.clone()
        x[0] = 0.0
        x[1] = 0.0
        x[1, 3] = 1e-30
        x[2] = torch.arange(x.shape[1]) % 3 - 1.0
        x[2, 0] = 2.54
        x[2, 1:5] = torch.tensor([0.01, -0.01, 1.27, -1.27])
        codes, scales = ops.quantize_int8(x.cuda())
        ref_c, ref_s = knn.quantize_int8(x.numpy())
        assert np.array_equal(codes.cpu().numpy(), ref_c)
        assert np.array_equal(scales.cpu().numpy(), ref_s)
        # the device form of the scale (a multiply by fp32(1/127)), not the CPU division
        assert np.array_equal(scales.cpu().numpy(), (x.cuda().abs().amax(1).clamp(min=1e-8) / 127.0).cpu().numpy())
