"""SilverTorch's bloom searches and the partial-mask scorer as ``torch.ops.st`` CUDA ops
(retrieve_b200/st_bloom.py, ``st.fused_kmean_ann_with_partial_masks``), against the
reference's own CPU searches (tests/golden/golden_bloom_st.npz, made by
tests/golden/make_golden_bloom_st.py) and the restatements in oracle/ivf.py."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ivf
from retrieve_b200 import _lib

BLOOM = np.load(Path(__file__).resolve().parent / "golden" / "golden_bloom_st.npz")
K, HASH_K = int(BLOOM["k"]), int(BLOOM["hash_k"])

PINNED = {  # retrieve/tests/parity/test_official.py:65-102; bloom_index_search.cpp:543-601
    "bloom_index_search_batch": (
        "st::bloom_index_search_batch(Tensor bloom_index, Tensor bloom_bundle_b_offsets, "
        "Tensor bloom_query_plans_data, Tensor bloom_query_plans_offsets, int k, int hash_k, "
        "bool return_bool_mask=True) -> Tensor"
    ),
    "bloom_index_search_batch_return_partial_response": (
        "st::bloom_index_search_batch_return_partial_response(Tensor bloom_index, "
        "Tensor bloom_bundle_b_offsets, Tensor bloom_query_plans_data, "
        "Tensor bloom_query_plans_offsets, Tensor selected_cluster_offsets, "
        "Tensor selected_cluster_lengths, int k, int hash_k, Tensor? query_plan_index=None) "
        "-> (Tensor, Tensor, Tensor)"
    ),
    "fused_kmean_ann_with_partial_masks": (
        "st::fused_kmean_ann_with_partial_masks(Tensor cluster_offsets, Tensor cluster_ids, "
        "Tensor cluster_length, Tensor embeddings, Tensor queries, int max_tensor_size_per_row, "
        "Tensor partial_mask_column_counts_cumsum, "
        "Tensor partial_mask_first_item_offset_in_column, "
        "Tensor partial_mask_column_results, int invalid_index_value=-1, int divisor_for_int8=-1, "
        "Tensor? filtering_bit_index=None, Tensor? per_embedding_scale=None, "
        "Tensor? cluster_warp_size=None, Tensor? cluster_warp_rounded_length_cumsum=None, "
        "Tensor? cluster_remaining_length_cumsum=None, Tensor? cluster_warp_size_cumsum=None, "
        "int total_cluster_rounded_warps=0, int total_cluster_remaining_warps=0) "
        "-> (Tensor, Tensor)"
    ),
    "bloom_index_search_batch_prepared": (
        "st::bloom_index_search_batch_prepared(Tensor bloom_index, Tensor bloom_bundle_b_offsets, "
        "Tensor plans, int plan_count, int max_stack_size, int k, int hash_k, "
        "bool return_bool_mask=False) -> Tensor"
    ),
    "bloom_index_search_batch_return_partial_response_prepared": (
        "st::bloom_index_search_batch_return_partial_response_prepared(Tensor bloom_index, "
        "Tensor bloom_bundle_b_offsets, Tensor plans, int plan_count, int max_stack_size, "
        "Tensor selected_cluster_offsets, Tensor selected_cluster_lengths, int k, int hash_k, "
        "Tensor? query_plan_index, int max_columns) -> (Tensor, Tensor, Tensor)"
    ),
    "fused_kmean_ann_with_partial_masks_multiple": (  # fused_kmean_ann.cpp:438-456
        "st::fused_kmean_ann_with_partial_masks_multiple(Tensor queries, Tensor[] list_cluster_offsets, "
        "Tensor[] list_selected_cluster_ids, Tensor[] list_selected_cluster_lengths, Tensor[] list_embeddings, "
        "int[] list_max_tensor_size_per_row, Tensor[] list_partial_mask_column_counts_cumsum, "
        "Tensor[] list_partial_mask_first_item_offset_in_column, Tensor[] list_partial_mask_column_results, "
        "int invalid_index_value=-1, int divisor_for_int8=-1, Tensor? filtering_bit_index=None, "
        "Tensor[]? list_per_embedding_scale=None, bool fuse=False) -> (Tensor[], Tensor[])"
    ),
    "bloom_index_search_batch_return_partial_response_multiple": (
        "st::bloom_index_search_batch_return_partial_response_multiple(Tensor[] list_bloom_index, "
        "Tensor[] list_bloom_bundle_b_offsets, Tensor bloom_query_plans_data, Tensor bloom_query_plans_offsets, "
        "Tensor[] list_selected_cluster_offsets, Tensor[] list_selected_cluster_lengths, int k, int hash_k, "
        "Tensor? query_plan_index=None, bool fuse=False) -> (Tensor[], Tensor[], Tensor[])"
    ),
    "generate_column_info_for_clusters": (
        "st::generate_column_info_for_clusters(Tensor selected_cluster_offsets, "
        "Tensor selected_cluster_lengths) -> (Tensor, Tensor, Tensor)"
    ),
}


def _st():
    import retrieve_b200.st  # noqa: F401  (registers the ops)

    return torch.ops.st


def _selection(probe_key="probe"):
    coff, sizes = BLOOM["cluster_offsets"], BLOOM["cluster_sizes"]
    probe = BLOOM[probe_key]
    return coff[probe].astype(np.int64), sizes[probe].astype(np.int64)


# --- CPU: the restatements pinned to the reference ----------------------------------------


def test_full_words_match_reference():
    words = ivf.bloom_full_words(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], BLOOM["plan_data"],
                                 BLOOM["plan_offsets"], K, HASH_K)
    assert np.array_equal(words, BLOOM["words"])
    n = int(BLOOM["n"])
    bits = np.unpackbits(BLOOM["words"].view(np.uint8).reshape(-1, 8)[:, ::-1], axis=1)
    bits = bits.reshape(BLOOM["words"].shape[0], -1)[:, :n]
    assert np.array_equal(bits, np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n])


def test_column_info_and_partial_response_match_reference():
    off, lens = _selection()
    counts, starts, first = ivf.column_info(off, lens)
    assert np.array_equal(counts, BLOOM["col_counts"]) and np.array_equal(starts, BLOOM["col_starts"])
    assert np.array_equal(first, BLOOM["col_first"])
    args = (BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], BLOOM["plan_data"], BLOOM["plan_offsets"])
    cumsum, first, words = ivf.bloom_partial_response(*args, off, lens, K, HASH_K)
    assert np.array_equal(cumsum, BLOOM["p_cumsum"]) and np.array_equal(first, BLOOM["p_first"])
    assert np.array_equal(words, BLOOM["p_words"])
    off2, lens2 = _selection("probe2")
    cumsum, first, words = ivf.bloom_partial_response(*args, off2, lens2, K, HASH_K, BLOOM["plan_index"])
    assert np.array_equal(cumsum, BLOOM["q_cumsum"]) and np.array_equal(first, BLOOM["q_first"])
    assert np.array_equal(words, BLOOM["q_words"])


def test_partial_scorer_restatement_equals_full_mask():
    """Over the probed ranges the partial response carries, the partial-mask scorer keeps what
    the full-N mask keeps (the reference's CPU scorer ignores the partial masks, so this
    property is the pin)."""
    rng = np.random.default_rng(2)
    off, lens = _selection()
    probe = BLOOM["probe"]
    n, d = int(BLOOM["n"]), 32
    codes = rng.integers(-127, 128, (n, d), dtype=np.int8)
    q = rng.integers(-127, 128, (probe.shape[0], d), dtype=np.int8)
    width = int(lens.sum(1).max())
    partial = (BLOOM["p_cumsum"], BLOOM["p_first"], BLOOM["p_words"])
    got = ivf.fused_kmean_ann(q, BLOOM["cluster_offsets"], probe, lens, codes, width, partial=partial)
    want = ivf.fused_kmean_ann(q, BLOOM["cluster_offsets"], probe, lens, codes, width,
                               filtering_bit_mask=BLOOM["words"])
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    assert (got[1] == -1).sum() > (ivf.fused_kmean_ann(q, BLOOM["cluster_offsets"], probe, lens, codes,
                                                       width)[1] == -1).sum()


def test_plan_stack_depth():
    from retrieve_b200.st_bloom import plan_stack_depth

    # the parser's own max_stack_size for the fixture's plans
    assert plan_stack_depth(BLOOM["plan_data"].view(np.uint8), BLOOM["plan_offsets"]) == int(BLOOM["max_stack"])


def test_schemas_are_the_reference_ones():
    st = _st()
    for name, schema in PINNED.items():
        assert str(getattr(st, name).default._schema) == schema, name


def test_fake_shapes():
    st = _st()
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        idx, boff = torch.empty(1000, dtype=torch.int64), torch.empty(4, dtype=torch.int64)
        out = st.bloom_index_search_batch_prepared(idx, boff, torch.empty(100, dtype=torch.int64), 6, 3, 5, 7)
        assert out.shape == (6, 96) and out.dtype == torch.int64
        out = st.bloom_index_search_batch_prepared(idx, boff, torch.empty(100, dtype=torch.int64), 6, 3, 5, 7, True)
        assert out.shape == (6, 96 * 64) and out.dtype == torch.bool
        sel = torch.empty(6, 4, dtype=torch.int64)
        c, s, f = st.generate_column_info_for_clusters(sel, sel)
        assert c.shape == s.shape == f.shape == (24,) and f.dtype == torch.int8
        cs, fi, w = st.bloom_index_search_batch_return_partial_response_prepared(
            idx, boff, torch.empty(100, dtype=torch.int64), 6, 3, sel, sel, 5, 7, None, 77)
        assert cs.shape == (24,) and cs.dtype == torch.int32 and w.shape == (77,)


def test_argument_errors_raise():
    _st()
    from retrieve_b200 import st_bloom

    with pytest.raises(RuntimeError, match="CUDA"):
        st_bloom.bloom_index_search_batch(torch.zeros(10, dtype=torch.int64), torch.zeros(2, dtype=torch.int64),
                                          torch.zeros(8, dtype=torch.int8), torch.zeros(8, dtype=torch.int64), 5, 7)
    with pytest.raises(RuntimeError, match="CUDA"):
        st_bloom.generate_column_info_for_clusters(torch.zeros(2, 3, dtype=torch.int64),
                                                   torch.zeros(2, 3, dtype=torch.int64))


def test_multiple_variants_check_their_lists():
    _st()
    from retrieve_b200 import st, st_bloom

    t = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="should not be empty"):
        st_bloom.bloom_index_search_batch_return_partial_response_multiple([], [], t, t, [], [], 5, 7)
    with pytest.raises(RuntimeError, match="same size"):
        st_bloom.bloom_index_search_batch_return_partial_response_multiple([t, t], [t], t, t, [t, t], [t, t], 5, 7)
    q = torch.zeros(2, 64, dtype=torch.int8)
    with pytest.raises(RuntimeError, match="list_embeddings must have the same size"):
        st.fused_kmean_ann_with_partial_masks_multiple(q, [t, t], [t, t], [t, t], [q], [8, 8], [t, t], [t, t], [t, t])


def test_capi_checks_need_no_device():
    lib = _lib.lib()
    fake = ctypes.c_void_p(16)  # never dereferenced: the checks fail first

    def search(k=5, hash_k=7, stack=3, plan_words=80, plan_count=10, index=fake):
        return lib.rb_st_bloom_search(index, 100, fake, 3, fake, plan_words, plan_count, stack, k, hash_k, 0, None,
                                      None)

    assert search(k=11) == _lib.RB_ERR_UNSUPPORTED
    assert search(stack=17) == _lib.RB_ERR_UNSUPPORTED
    assert search(k=0) == _lib.RB_ERR_INVALID_ARG
    assert search(plan_words=79) == _lib.RB_ERR_INVALID_ARG
    assert search(index=None) == _lib.RB_ERR_INVALID_ARG
    assert search() == _lib.RB_ERR_INVALID_ARG  # null output
    assert search(plan_count=0) == _lib.RB_OK
    assert lib.rb_st_bloom_column_info(None, None, -1, None, None, None, None, None) == _lib.RB_ERR_INVALID_ARG
    assert lib.rb_st_bloom_column_info(None, None, 0, None, None, None, None, None) == _lib.RB_OK
    assert lib.rb_st_bloom_partial_search(fake, 100, fake, 3, fake, 80, 10, 3, None, 4, 2, None, None, 5, 7, fake,
                                          10, None) == _lib.RB_ERR_INVALID_ARG  # ranges without their cumsum
    assert lib.rb_st_bloom_partial_search(fake, 100, fake, 3, fake, 80, 10, 3, None, 4, 2, fake, fake, 5, 7, None,
                                          0, None) == _lib.RB_OK  # no words asked
    assert lib.rb_st_fused_kmean_ann_with_partial_masks(
        None, 8, None, None, 2, None, 100, None, _lib.RB_I8, 4, 64, 90, None, None, None, 0, 4, None, None, -1, -1,
        None, None, None, 0, None) == _lib.RB_ERR_INVALID_ARG  # ranges without their cumsum
    assert lib.rb_st_fused_kmean_ann_with_partial_masks(
        None, 8, None, None, 2, None, 100, None, _lib.RB_I8, 4, 64, 90, fake, fake, None, 0, 3, None, None, -1, -1,
        None, None, None, 0, None) == _lib.RB_ERR_INVALID_ARG  # 3 mask rows for 4 query rows, no filtering_bit_index


# --- GPU -----------------------------------------------------------------------------------


def _dev(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


@pytest.mark.gpu
def test_full_search_on_device():
    """Packed words and bool masks equal the reference's CPU search, from the parser's plans
    and from the prepared blob (with spare plan slots)."""
    st = _st()
    index, boff, data, offs = _dev(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], BLOOM["plan_data"],
                                   BLOOM["plan_offsets"])
    words = st.bloom_index_search_batch(index, boff, data, offs, K, HASH_K, False)
    assert np.array_equal(words.cpu().numpy(), BLOOM["words"])
    mask = st.bloom_index_search_batch(index, boff, data.cpu(), offs.cpu(), K, HASH_K)
    n = int(BLOOM["n"])
    assert mask.dtype == torch.bool
    assert np.array_equal(mask.cpu().numpy()[:, :n], np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n].astype(bool))
    # the adapter's blob holds `slots` plan slots and passes `slots` as plan_count; the data
    # follows the 8 * slots offset words (adapter.py:219-236), the spare slots' offsets are zero
    n_plans = BLOOM["words"].shape[0]
    slots = n_plans + 3
    blob = torch.from_numpy(ivf.plan_blob(BLOOM["plan_data"], BLOOM["plan_offsets"], slots)).cuda()
    words_p = st.bloom_index_search_batch_prepared(index, boff, blob, slots, int(BLOOM["max_stack"]), K, HASH_K)
    assert words_p.shape[0] == slots
    assert np.array_equal(words_p[:n_plans].cpu().numpy(), BLOOM["words"])
    mask_p = st.bloom_index_search_batch_prepared(index, boff, blob, slots, int(BLOOM["max_stack"]), K, HASH_K,
                                                  True)
    assert torch.equal(mask_p[:n_plans], mask)


@pytest.mark.gpu
def test_column_info_and_partial_response_on_device():
    st = _st()
    index, boff, data, offs = _dev(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], BLOOM["plan_data"],
                                   BLOOM["plan_offsets"])
    off, lens = _dev(*_selection())
    c, s, f = st.generate_column_info_for_clusters(off, lens)
    assert np.array_equal(c.cpu().numpy(), BLOOM["col_counts"]) and np.array_equal(s.cpu().numpy(), BLOOM["col_starts"])
    assert np.array_equal(f.cpu().numpy(), BLOOM["col_first"])
    cumsum, first, words = st.bloom_index_search_batch_return_partial_response(index, boff, data, offs, off, lens, K,
                                                                               HASH_K)
    for got, key in ((cumsum, "p_cumsum"), (first, "p_first"), (words, "p_words")):
        assert got.dtype == torch.from_numpy(BLOOM[key]).dtype and np.array_equal(got.cpu().numpy(), BLOOM[key]), key
    off2, lens2, plan_index = _dev(*_selection("probe2"), BLOOM["plan_index"])
    cumsum, first, words = st.bloom_index_search_batch_return_partial_response(index, boff, data, offs, off2, lens2,
                                                                               K, HASH_K, plan_index)
    for got, key in ((cumsum, "q_cumsum"), (first, "q_first"), (words, "q_words")):
        assert np.array_equal(got.cpu().numpy(), BLOOM[key]), key
    # prepared: a static capacity with a zero tail, rows mapped to plan slots by the index
    n_plans = BLOOM["words"].shape[0]
    blob = torch.from_numpy(ivf.plan_blob(BLOOM["plan_data"], BLOOM["plan_offsets"], n_plans)).cuda()
    cap = BLOOM["q_words"].size + 37
    cumsum, first, words = st.bloom_index_search_batch_return_partial_response_prepared(
        index, boff, blob, n_plans, int(BLOOM["max_stack"]), off2, lens2, K, HASH_K, plan_index, cap)
    assert np.array_equal(cumsum.cpu().numpy(), BLOOM["q_cumsum"])
    w = words.cpu().numpy()
    assert w.shape == (cap,) and np.array_equal(w[: BLOOM["q_words"].size], BLOOM["q_words"]) and not w[-37:].any()


@pytest.mark.gpu
@pytest.mark.parametrize("divisor", [-1, 16])
def test_fused_kmean_ann_with_partial_masks(divisor):
    """The reference's partial response drives the partial-mask scorer: equal to the
    restatement and to fused_kmean_ann under the full-N packed words, bit for bit."""
    st = _st()
    rng = np.random.default_rng(5)
    off, lens = _selection()
    probe = BLOOM["probe"]
    n, d = int(BLOOM["n"]), 64
    codes = rng.integers(-127, 128, (n, d), dtype=np.int8)
    q = rng.integers(-127, 128, (probe.shape[0], d), dtype=np.int8)
    width = int(lens.sum(1).max())
    t = _dev(BLOOM["cluster_offsets"], probe, lens, codes, q)
    partial = _dev(BLOOM["p_cumsum"], BLOOM["p_first"], BLOOM["p_words"])
    raw, idx = st.fused_kmean_ann_with_partial_masks(*t, width, *partial, invalid_index_value=-2,
                                                     divisor_for_int8=divisor)
    want_r, want_i = ivf.fused_kmean_ann(q, BLOOM["cluster_offsets"], probe, lens, codes, width,
                                         divisor_for_int8=divisor, invalid_index_value=-2,
                                         partial=(BLOOM["p_cumsum"], BLOOM["p_first"], BLOOM["p_words"]))
    raw_np = raw.cpu().numpy()
    if divisor != -1:
        raw_np, want_r = raw_np.view(np.uint16), want_r.view(np.uint16)
    assert np.array_equal(raw_np, want_r) and np.array_equal(idx.cpu().numpy(), want_i)
    full_r, full_i = st.fused_kmean_ann(*t, width, filtering_bit_mask=torch.from_numpy(BLOOM["words"]).cuda(),
                                        invalid_index_value=-2, divisor_for_int8=divisor)
    assert torch.equal(full_i, idx) and torch.equal(full_r.view(torch.int16) if divisor != -1 else full_r,
                                                    raw.view(torch.int16) if divisor != -1 else raw)


@pytest.mark.gpu
def test_multiple_variants_equal_their_single_ops():
    """The chunked-index variants: one result per chunk, each equal to the single op on that
    chunk (the reference's loop; fuse changes nothing), here with the index given twice and two
    different probe selections."""
    st = _st()
    index, boff, data, offs = _dev(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], BLOOM["plan_data"],
                                   BLOOM["plan_offsets"])
    off_a, len_a = _dev(*_selection())
    rows = BLOOM["probe"].shape[0]
    probe_b = BLOOM["probe2"][:rows]
    off_b = torch.from_numpy(BLOOM["cluster_offsets"][probe_b].astype(np.int64)).cuda()
    len_b = torch.from_numpy(BLOOM["cluster_sizes"][probe_b].astype(np.int64)).cuda()
    for fuse in (False, True):
        cs, fi, ws = st.bloom_index_search_batch_return_partial_response_multiple(
            [index, index], [boff, boff], data, offs, [off_a, off_b], [len_a, len_b], K, HASH_K, None, fuse)
        for c, (o, ln) in enumerate(((off_a, len_a), (off_b, len_b))):
            want = ivf.bloom_partial_response(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], BLOOM["plan_data"],
                                              BLOOM["plan_offsets"], o.cpu().numpy(), ln.cpu().numpy(), K, HASH_K)
            for got, w in zip((cs[c], fi[c], ws[c]), want):
                assert np.array_equal(got.cpu().numpy(), w)
    rng = np.random.default_rng(9)
    n, d = int(BLOOM["n"]), 64
    codes = torch.from_numpy(rng.integers(-127, 128, (n, d), dtype=np.int8)).cuda()
    q = torch.from_numpy(rng.integers(-127, 128, (rows, d), dtype=np.int8)).cuda()
    coff = torch.from_numpy(BLOOM["cluster_offsets"]).cuda()
    ids = [torch.from_numpy(BLOOM["probe"]).cuda(), torch.from_numpy(probe_b.astype(np.int64)).cuda()]
    widths = [int(len_a.sum(1).max()), int(len_b.sum(1).max())]
    raws, idxs = st.fused_kmean_ann_with_partial_masks_multiple(
        q, [coff, coff], ids, [len_a, len_b], [codes, codes], widths, cs, fi, ws, -1, 16)
    for c in range(2):
        raw, idx = st.fused_kmean_ann_with_partial_masks(coff, ids[c], [len_a, len_b][c], codes, q, widths[c], cs[c],
                                                         fi[c], ws[c], -1, 16)
        assert torch.equal(raws[c], raw) and torch.equal(idxs[c], idx)


# The reference's known answers for its bloom path (retrieve/tests/parity/test_official.py:229-245,
# 355-373, 414-430, 515-522): a 4-doc corpus with 2 features (language; category), its index at
# b_multiplier 5.0 and 3 positions a value, three expressions parsed with 7 stored hashes a term.
README_CORPUS = np.array([
    [[100, -1], [200, 201]],  # doc 0: en; music, pop
    [[100, 101], [200, -1]],  # doc 1: en, es; music
    [[102, -1], [202, -1]],  # doc 2: ja; news
    [[100, -1], [200, 203]],  # doc 3: en; music, rock
])
README_QUERIES = ["0:100", "0:100 AND NOT 1:201", "0:102 OR 1:203"]
README_HITS = [[0, 1, 3], [1, 3], [2, 3]]


def _readme_plans():
    _st()
    _, (data, offsets) = torch.ops.st.parse_expression_query_batch(
        README_QUERIES + [""], torch.ones(4, dtype=torch.int64), 7, True, 5)
    return data.numpy(), offsets.numpy()


def test_readme_known_answers_on_the_restatement():
    """The library's parser and the restated bloom build and search give the reference's hits,
    the match-all empty expression, and its partial response over two 2-doc ranges."""
    fid, foff, fval = ivf.attrs_to_features(README_CORPUS)
    index, boff = ivf.bloom_index_build(fid, foff, fval, 5.0, 3)
    assert len(boff) == 2  # one 2048-doc bundle
    data, offsets = _readme_plans()
    for p, hits in enumerate(README_HITS + [[0, 1, 2, 3]]):
        mask = ivf.bloom_plan_mask(index, boff, data, offsets, p, 3, 7, 4)
        assert np.nonzero(mask)[0].tolist() == hits
    sel_off, sel_len = np.array([[0, 2]] * 3), np.array([[2, 2]] * 3)
    cumsum, first, words = ivf.bloom_partial_response(index, boff, data, offsets[:24], sel_off, sel_len, 3, 7)
    assert cumsum.tolist() == [1, 2, 3, 4, 5, 6] and first.tolist() == [0, 2] * 3
    for r, hits in enumerate(README_HITS):
        kept = [2 * j + i for j in range(2) for i in range(2)
                if ivf.partial_mask_keep(cumsum, first, words, r * 2 + j, np.array([i]))[0]]
        assert sorted(kept) == hits


@pytest.mark.gpu
def test_readme_known_answers_on_the_device():
    st = _st()
    fid, foff, fval = (torch.from_numpy(np.ascontiguousarray(a)).cuda()
                       for a in ivf.attrs_to_features(README_CORPUS))
    index, boff = st.bloom_index_build(fid, foff, fval, 5.0, 3)
    data, offsets = (torch.from_numpy(a) for a in _readme_plans())
    full = st.bloom_index_search_batch(index, boff, data, offsets, 3, 7, True)
    assert full.dtype == torch.bool and full.shape == (4, 2048)
    for row, hits in zip(full[:, :4].cpu().tolist(), README_HITS + [[0, 1, 2, 3]]):
        assert [i for i, h in enumerate(row) if h] == hits
    packed = st.bloom_index_search_batch(index, boff, data, offsets, 3, 7, False)
    assert packed.shape == (4, 32)
    assert np.array_equal(packed.cpu().numpy(), ivf.pack_mask_high_first(full.cpu().numpy()))
    sel_off = torch.tensor([[0, 2]] * 3).cuda()
    sel_len = torch.tensor([[2, 2]] * 3).cuda()
    cumsum, first, words = st.bloom_index_search_batch_return_partial_response(
        index, boff, data, offsets[:24], sel_off, sel_len, 3, 7)
    assert cumsum.tolist() == [1, 2, 3, 4, 5, 6] and first.tolist() == [0, 2] * 3


def _expressions(query_attrs, reverse):
    """The adapter's AND-only expressions (retrieve/src/retrieve/ops/official/adapter.py:127-157):
    one ``c:v`` term per active clause, ``NOT`` on reversed clauses, "" when none is active."""
    out = []
    for row in np.asarray(query_attrs).tolist():
        terms = [("NOT " if reverse[c] else "") + f"{c}:{v}" for c, v in enumerate(row) if v != -1]
        out.append(" AND ".join(terms))
    return out


def _bloom_corpus(seed=7, n=6000, c=2, a_max=3, vocab=50):
    rng = np.random.default_rng(seed)
    attrs = rng.integers(0, vocab, (n, c, a_max))
    attrs[rng.random((n, c, a_max)) < 0.4] = -1
    return attrs


def test_bloom_keeps_every_exact_match_and_not_flips_the_guarantee():
    """The reference's T4 properties (test_official.py:455-508) on the restatement with the
    library's parser: an AND of terms never loses a doc the exact predicate accepts and lets
    through under 5 % of the rest at b_multiplier 10; a single NOT term never admits a doc that
    holds the value."""
    from oracle import filters

    attrs = _bloom_corpus()
    n, c, _ = attrs.shape
    fid, foff, fval = ivf.attrs_to_features(attrs)
    index, boff = ivf.bloom_index_build(fid, foff, fval, 10.0, K)
    rng = np.random.default_rng(42)
    qa = rng.integers(0, 50, (16, c))
    _st()
    for reverse in ([False, False], [True, False]):
        q = qa.copy()
        if reverse[0]:
            q[:, 1] = -1
        exprs = _expressions(q, reverse)
        _, (data, offsets) = torch.ops.st.parse_expression_query_batch(exprs, torch.ones(len(exprs)), HASH_K, True, 5)
        bloom = np.stack([ivf.bloom_plan_mask(index, boff, data.numpy(), offsets.numpy(), p, K, HASH_K, n)
                          for p in range(len(exprs))])
        exact = filters.clause_mask(attrs, np.array(reverse), q)
        if not reverse[0]:
            assert not (exact & ~bloom).any(), "the bloom lost an exact match"
            assert (bloom & ~exact).sum() / max((~exact).sum(), 1) < 0.05
        else:
            assert not (bloom & ~exact).any(), "a bloom NOT admitted a doc holding the value"


@pytest.mark.gpu
def test_bloom_properties_on_the_device():
    """The same on the device build and search, which equal the restatement's masks."""
    from oracle import filters

    st = _st()
    attrs = _bloom_corpus(seed=9)
    n, c, _ = attrs.shape
    fid, foff, fval = ivf.attrs_to_features(attrs)
    index, boff = st.bloom_index_build(*(torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (fid, foff, fval)),
                                       10.0, K)
    rng = np.random.default_rng(43)
    qa = rng.integers(0, 50, (16, c))
    exprs = _expressions(qa, [False, False])
    _, (data, offsets) = torch.ops.st.parse_expression_query_batch(exprs, torch.ones(len(exprs)), HASH_K, True, 5)
    full = st.bloom_index_search_batch(index, boff, data, offsets, K, HASH_K, True)[:, :n].cpu().numpy()
    exact = filters.clause_mask(attrs, np.zeros(c, dtype=bool), qa)
    assert not (exact & ~full).any()
    assert (full & ~exact).sum() / max((~exact).sum(), 1) < 0.05
    want_index, want_boff = ivf.bloom_index_build(fid, foff, fval, 10.0, K)
    assert np.array_equal(index.cpu().numpy(), want_index) and np.array_equal(boff.cpu().numpy(), want_boff)


@pytest.mark.gpu
def test_prepared_ops_replay_in_a_cuda_graph():
    """The prepared bloom searches and the raw scorers never wait on the host, so they capture into
    a CUDA graph: replays after new inputs are copied in equal eager calls."""
    st = _st()
    index, boff = _dev(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"])
    n_plans = BLOOM["words"].shape[0]
    blob = torch.from_numpy(ivf.plan_blob(BLOOM["plan_data"], BLOOM["plan_offsets"], n_plans)).cuda()
    off, lens = _dev(*_selection())
    rng = np.random.default_rng(4)
    n, d = int(BLOOM["n"]), 64
    codes = torch.from_numpy(rng.integers(-127, 128, (n, d), dtype=np.int8)).cuda()
    q = torch.from_numpy(rng.integers(-127, 128, (off.shape[0], d), dtype=np.int8)).cuda()
    coff = torch.from_numpy(BLOOM["cluster_offsets"]).cuda()
    probe = torch.from_numpy(BLOOM["probe"]).cuda()
    width = int(lens.sum(1).max())
    cap = int(BLOOM["p_words"].size) + 64

    def call():
        words = st.bloom_index_search_batch_prepared(index, boff, blob, n_plans, int(BLOOM["max_stack"]), K, HASH_K)
        cs, fi, pw = st.bloom_index_search_batch_return_partial_response_prepared(
            index, boff, blob, n_plans, int(BLOOM["max_stack"]), off, lens, K, HASH_K, None, cap)
        raw, idx = st.fused_kmean_ann_with_partial_masks(coff, probe, lens, codes, q, width, cs, fi, pw)
        return words, pw, raw, idx

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            call()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = call()
    for seed in range(2):
        q.copy_(torch.from_numpy(np.random.default_rng(seed).integers(-127, 128, tuple(q.shape), dtype=np.int8)))
        graph.replay()
        want = call()
        torch.cuda.synchronize()
        for a, b in zip(outs, want):
            assert torch.equal(a, b)
    del graph
