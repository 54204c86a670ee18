"""Filtered dense top-k (BASELINE config 3 semantics) against the oracle:
integer-valued embeddings make every score exact, so ids and scores match bit
for bit, ties toward the lower id; exact, Bloom and Bloom+recheck predicates;
the device Bloom build equals the oracle's (pinned to the reference's own
build)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bloom, predicate
from oracle.dense import as_f32
from oracle.select import topk_strict
from retrieve_b200 import predicates as P
from tests.golden import golden_inputs as gi
from tests.helpers import assert_topk_exact, make_int_rows

pytestmark = pytest.mark.gpu

EXPRS = gi.BLOOM_EXPRESSIONS


def _oracle(q, x, k, masks):
    sc = as_f32(q) @ as_f32(x).T
    return topk_strict(sc, k, valid=masks, sentinel=True)


def _masks(exprs, b, attrs=None, words=None):
    return np.stack([predicate.eval_items(predicate.parse(exprs[i % len(exprs)]), attrs=attrs, words=words)
                     for i in range(b)])


def test_bloom_build_matches_oracle():
    from retrieve_b200 import ops

    attrs = gi.zipf_attrs(5000, seed=3)
    words = ops.bloom_build(attrs[:, :, None].contiguous().cuda(), 3).cpu().numpy().view(np.uint64)
    assert np.array_equal(words, bloom.item_words(attrs.numpy(), k=3))


@pytest.mark.parametrize("mode", ["exact", "bloom", "bloom_recheck"])
@pytest.mark.parametrize("b,n,k", [(64, 20_000, 50), (300, 60_000, 100), (130, 400_000, 100)])
def test_filtered_topk_exact(mode, b, n, k):
    from retrieve_b200 import ops

    attrs = gi.zipf_attrs(n, seed=n)
    attrs3 = attrs[:, :, None].contiguous()
    q = make_int_rows(b, 128, seed=1)
    x = make_int_rows(n, 128, seed=2)
    exprs = [EXPRS[i % len(EXPRS)] for i in range(b)]
    preds = P.from_expressions(exprs).to("cuda")
    words = ops.bloom_build(attrs3.cuda(), 3)
    ids, scores = ops.dense_topk_filtered(q.cuda(), x.cuda(), k, preds.terms, preds.n_terms, mode,
                                          attrs3.cuda(), words)
    wn = words.cpu().numpy().view(np.uint64)
    if mode == "exact":
        masks = _masks(exprs, b, attrs=attrs.numpy())
    elif mode == "bloom":
        masks = _masks(exprs, b, words=wn)
    else:
        masks = _masks(exprs, b, attrs=attrs.numpy()) & _masks(exprs, b, words=wn)
    ref_ids, ref_scores = _oracle(q, x, k, masks)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


@pytest.mark.parametrize("mode", ["exact", "bloom_recheck"])
@pytest.mark.parametrize("b,n,k", [(200, 400_000, 10), (130, 1_000_000, 100)])
def test_speculative_seed_and_second_pass(mode, b, n, k):
    """Corpora large enough for a sampled seed: the full pass starts from the speculative
    seed (the ceil(3k / s)-th sampled chunk max); rows that come back with fewer than k
    results (a value no item holds, a rare conjunction, an unlucky sample) run again from
    the safe seed. Bit for bit the oracle's either way."""
    from retrieve_b200 import ops

    attrs = gi.zipf_attrs(n, seed=n + 1)
    attrs3 = attrs[:, :, None].contiguous()
    q = make_int_rows(b, 128, seed=7)
    x = make_int_rows(n, 128, seed=8)
    exprs = [EXPRS[i % len(EXPRS)] for i in range(b)]
    for r in range(0, b, 9):
        exprs[r] = "0:12345"  # no item holds the value
    for r in range(4, b, 9):
        exprs[r] = "5:0 AND 6:1 AND 7:2 AND 1:3"  # a few hundred items at most
    preds = P.from_expressions(exprs).to("cuda")
    words = ops.bloom_build(attrs3.cuda(), 3)
    ids, scores = ops.dense_topk_filtered(q.cuda(), x.cuda(), k, preds.terms, preds.n_terms, mode,
                                          attrs3.cuda(), words)
    masks = _masks(exprs, b, attrs=attrs.numpy())
    if mode == "bloom_recheck":
        masks &= _masks(exprs, b, words=words.cpu().numpy().view(np.uint64))
    assert not masks[0].any()
    ref_ids, ref_scores = _oracle(q, x, k, masks)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


def test_linr_clause_queries_filtered():
    """LiNR V1 semantics: AND of clause values with reverse clauses."""
    from oracle import filters
    from retrieve_b200 import ops

    b, n, k = 96, 30_000, 64
    g = torch.Generator().manual_seed(4)
    attrs = torch.randint(0, 5, (n, 4, 2), generator=g)
    attrs[torch.rand(n, 4, 2, generator=g) < 0.3] = -1
    qa = torch.randint(0, 5, (b, 4), generator=g)
    qa[torch.rand(b, 4, generator=g) < 0.4] = -1
    rev = torch.tensor([False, False, True, False])
    preds = P.from_clause_attrs(qa, rev).to("cuda")
    q, x = make_int_rows(b, 128, seed=3), make_int_rows(n, 128, seed=4)
    ids, scores = ops.dense_topk_filtered(q.cuda(), x.cuda(), k, preds.terms, preds.n_terms, "exact",
                                          attrs.cuda(), None)
    ref_ids, ref_scores = _oracle(q, x, k, filters.clause_mask(attrs.numpy(), rev.numpy(), qa.numpy()))
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


@pytest.mark.parametrize("mode", ["bloom", "bloom_recheck"])
def test_sliced_bloom_test_equals_the_per_item_test(mode):
    """The Bloom words bit-sliced (a workspace of rb_dense_topk_filtered_workspace_size) and
    tested item by item (a workspace of rb_dense_topk_workspace_size) give the same top-k;
    rows whose terms split a group (the per-item test on those queries) too."""
    import ctypes

    from retrieve_b200 import _lib, ops

    b, n, k = 200, 50_000, 100
    attrs = gi.zipf_attrs(n, seed=11)
    attrs3 = attrs[:, :, None].contiguous().cuda()
    q, x = make_int_rows(b, 128, seed=5).cuda(), make_int_rows(n, 128, seed=6).cuda()
    exprs = [EXPRS[i % len(EXPRS)] for i in range(b)]
    preds = P.from_expressions(exprs)
    terms = preds.terms.clone()
    rec = terms.view(b, 8, 24)
    nt = preds.n_terms
    for r in range(0, b, 7):  # rotate a row's terms: a group's terms are then not contiguous
        if nt[r] >= 3:
            rec[r, : nt[r]] = torch.roll(rec[r, : nt[r]].clone(), 1, dims=0)
    terms, nt = terms.cuda(), nt.to(torch.int32).cuda()
    words = ops.bloom_build(attrs3, 3)
    m = ops.FILTER_MODES[mode]
    lib = _lib.lib()
    f = ops._RbFilter(m, terms.data_ptr(), nt.data_ptr(), attrs3.data_ptr(), attrs3.shape[1], attrs3.shape[2],
                      words.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = []
    for sliced in (False, True):
        nb = ctypes.c_size_t(0)
        if sliced:
            _lib.check(lib.rb_dense_topk_filtered_workspace_size(b, n, 128, _lib.RB_BF16, k, m, ctypes.byref(nb)),
                       "ws")
        else:
            _lib.check(lib.rb_dense_topk_workspace_size(b, n, 128, _lib.RB_BF16, k, ctypes.byref(nb)), "ws")
        ws = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
        ids = torch.empty(b, k, dtype=torch.int64, device="cuda")
        sc = torch.empty(b, k, dtype=torch.float32, device="cuda")
        _lib.check(lib.rb_dense_topk_filtered(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(x.data_ptr()), b, n, 128,
                                              _lib.RB_BF16, k, 0, ctypes.addressof(f), ctypes.c_void_p(ids.data_ptr()),
                                              ctypes.c_void_p(sc.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nb.value,
                                              stream), "filtered")
        out.append((ids.cpu().numpy(), sc.cpu().numpy()))
    assert np.array_equal(out[0][1], out[1][1]) and np.array_equal(out[0][0], out[1][0])
    wn = words.cpu().numpy().view(np.uint64)
    masks = _masks(exprs, b, words=wn)
    if mode == "bloom_recheck":
        masks &= _masks(exprs, b, attrs=attrs.numpy())
    ref_ids, ref_scores = _oracle(q.cpu(), x.cpu(), k, masks)
    assert_topk_exact(out[1][0], out[1][1], ref_ids, ref_scores)


@pytest.mark.parametrize("layout", ["two_values", "odd_row", "unaligned"])
@pytest.mark.parametrize("mode", ["exact", "bloom_recheck"])
def test_attribute_rows_outside_the_ring(layout, mode):
    """The 2-SM filtered kernel (B > 128) streams attribute rows of at most 8 cells, a whole
    number of 16-byte units at a 16-byte aligned address, through its shared-memory ring;
    other rows are rechecked from global memory: 16 cells (8 clauses x 2 values), 5 cells
    (an odd row) and 8 cells at an address 8 bytes off alignment. Bit for bit the oracle's."""
    from retrieve_b200 import ops

    b, n, k = 260, 80_000, 50
    base = gi.zipf_attrs(n, seed=21)
    if layout == "two_values":
        second = gi.zipf_attrs(n, seed=22)
        second[torch.rand(n, 8, generator=torch.Generator().manual_seed(5)) < 0.5] = -1
        attrs3 = torch.stack([base, second], dim=2).contiguous()  # [n, 8, 2]
        exprs = [EXPRS[i % len(EXPRS)] for i in range(b)]
    elif layout == "odd_row":
        attrs3 = base[:, :5, None].contiguous()  # [n, 5, 1]
        exprs = ["0:0", "1:3 OR 2:7", "0:1 AND 3:2", "NOT 0:0", "(4:5 OR 1:1) AND 0:2", "1:0 AND NOT 2:0"]
        exprs = [exprs[i % len(exprs)] for i in range(b)]
    else:
        attrs3 = base[:, :, None].contiguous()
        exprs = [EXPRS[i % len(EXPRS)] for i in range(b)]
    q = make_int_rows(b, 128, seed=23)
    x = make_int_rows(n, 128, seed=24)
    preds = P.from_expressions(exprs).to("cuda")
    dev_attrs = attrs3.cuda()
    if layout == "unaligned":
        flat = torch.empty(attrs3.numel() + 1, dtype=torch.int64, device="cuda")
        flat[1:] = dev_attrs.reshape(-1)
        dev_attrs = flat[1:].view(attrs3.shape)  # 8 bytes past a 16-byte boundary
        assert dev_attrs.data_ptr() % 16 == 8
    words = ops.bloom_build(dev_attrs, 3)
    ids, scores = ops.dense_topk_filtered(q.cuda(), x.cuda(), k, preds.terms, preds.n_terms, mode, dev_attrs, words)
    masks = _masks(exprs, b, attrs=attrs3.numpy())
    if mode == "bloom_recheck":
        masks &= _masks(exprs, b, words=words.cpu().numpy().view(np.uint64))
    ref_ids, ref_scores = _oracle(q, x, k, masks)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


@pytest.mark.parametrize("b", [64, 300])
@pytest.mark.parametrize("mode", ["bloom", "bloom_recheck"])
def test_prebuilt_bloom_slices_equal_per_call_build(mode, b):
    """Bloom words bit-sliced once at build time (``bloom_slices``) and passed to the search give
    the same top-k as the slices the call builds into its workspace (1-SM and 2-SM kernels)."""
    from retrieve_b200 import ops

    n, k = 90_000, 40
    attrs = gi.zipf_attrs(n, seed=41)[:, :, None].contiguous().cuda()
    q = make_int_rows(b, 128, seed=42).cuda()
    x = make_int_rows(n, 128, seed=43).cuda()
    exprs = [EXPRS[i % len(EXPRS)] for i in range(b)]
    preds = P.from_expressions(exprs).to("cuda")
    words = ops.bloom_build(attrs, 3)
    slices = ops.bloom_slices(words)
    assert slices.numel() == (n + 127) // 128 * 256
    ids0, sc0 = ops.dense_topk_filtered(q, x, k, preds.terms, preds.n_terms, mode, attrs, words)
    ids1, sc1 = ops.dense_topk_filtered(q, x, k, preds.terms, preds.n_terms, mode, attrs, words, slices)
    assert torch.equal(ids0, ids1)
    assert torch.equal(sc0, sc1)
