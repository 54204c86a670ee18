"""Pins the ``st::search`` restatement (oracle/ivf.py) to the reference: the
fixture made by the reference's adapter epilogue over its own CPU scorer
(tests/golden/make_golden_ivf.py), and the slot-order and prep facts of the
reference's CUDA op. CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import ivf, knn
from tests.helpers import assert_topk_equal_up_to_ties

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden_ivf.npz")
N_CASES = len({k.split("_")[0] for k in GOLDEN.files})


def _case(ci):
    p = f"c{ci}_"
    g = {k[len(p):]: GOLDEN[k] for k in GOLDEN.files if k.startswith(p)}
    n_lists, max_size, n_probe, d, k, b, width, div, ties = g["shape"].tolist()
    return g, dict(k=k, width=width, div=div, d=d, b=b)


def _args(g, meta):
    return (g["query"], g["probe"], g["offsets"], g["sizes"], g["codes"], g["sort_perm"], g["gs"],
            meta["k"], meta["width"])


def _check(ids, scores, ref_ids, ref_scores):
    assert_topk_equal_up_to_ties(ids, scores, ref_ids, ref_scores)
    pad = np.isneginf(ref_scores)
    assert (ids[pad] == -1).all() and (ref_ids[pad] == -1).all()


@pytest.mark.parametrize("ci", range(N_CASES))
def test_int32_path_matches_reference(ci):
    g, meta = _case(ci)
    ids, scores = ivf.search(*_args(g, meta))
    _check(ids, scores, g["ids32"], g["sc32"])


@pytest.mark.parametrize("ci", range(N_CASES))
def test_fp16_path_matches_reference(ci):
    g, meta = _case(ci)
    assert meta["div"] == ivf.default_divisor(meta["d"])
    ids, scores = ivf.search(*_args(g, meta), divisor_for_int8=meta["div"])
    _check(ids, scores, g["ids16"], g["sc16"])


@pytest.mark.parametrize("ci", range(N_CASES))
def test_filter_mask_matches_reference(ci):
    """The fixture's boolean mask, packed high bit first as the CUDA scorer reads it
    (the CPU run got it packed low bit first, the CPU scorer's order)."""
    g, meta = _case(ci)
    words = ivf.pack_mask_high_first(g["mask"])
    ids, scores = ivf.search(*_args(g, meta), filtering_bit_mask=words)
    _check(ids, scores, g["idsm"], g["scm"])
    kept = ids >= 0
    rows = np.nonzero(kept)[0]
    inv = np.argsort(g["sort_perm"])
    assert g["mask"][rows, inv[ids[kept]]].all(), "a filtered-out position was returned"


@pytest.mark.parametrize("ci", range(N_CASES))
def test_raw_dots_match_reference_scorer(ci):
    """The scorer's raw row (st.fused_kmean_ann on the CPU): the same (position, int32
    dot) multiset as the restatement's slots, INT32_MIN / -1 in the pad slots."""
    g, meta = _case(ci)
    codes, _ = knn.quantize_int8(g["query"])
    raw, idx = g["raw"], g["idx"]
    assert raw.shape == (meta["b"], ivf.padded_width(meta["width"])) and raw.dtype == np.int32
    for r in range(meta["b"]):
        pos = ivf.probe_slots(g["probe"][r], g["offsets"], g["sizes"])
        dots = ivf.raw_scores(codes[r], g["codes"], pos, -1)
        valid = idx[r] >= 0
        assert (raw[r][~valid] == ivf.INT32_MIN).all()
        got = sorted(zip(idx[r][valid].tolist(), raw[r][valid].tolist()))
        assert got == sorted(zip(pos.tolist(), dots.tolist()))


@pytest.mark.parametrize("ci", range(N_CASES))
def test_fused_kmean_ann_rows_match_reference_scorer(ci):
    """``ivf.fused_kmean_ann`` (the CUDA op's row, slot order and pads) holds per row the
    same (position, raw) multiset as the reference's CPU scorer, whose rows follow probe
    order; the fp16 path's raws are the int32 dots divided and rounded."""
    g, meta = _case(ci)
    codes, _ = knn.quantize_int8(g["query"])
    lengths = g["sizes"][g["probe"]]
    raw, idx = ivf.fused_kmean_ann(codes, g["offsets"], g["probe"], lengths, g["codes"], meta["width"])
    assert raw.shape == g["raw"].shape and raw.dtype == np.int32 and idx.dtype == np.int32
    for r in range(meta["b"]):
        valid = g["idx"][r] >= 0
        want = sorted(zip(g["idx"][r][valid].tolist(), g["raw"][r][valid].tolist()))
        assert sorted(zip(idx[r][idx[r] >= 0].tolist(), raw[r][idx[r] >= 0].tolist())) == want
        assert (raw[r][idx[r] < 0] == ivf.INT32_MIN).all()
    r16, i16 = ivf.fused_kmean_ann(codes, g["offsets"], g["probe"], lengths, g["codes"], meta["width"],
                                   divisor_for_int8=meta["div"], invalid_index_value=-7)
    assert r16.dtype == np.float16 and (i16 == np.where(idx >= 0, idx, -7)).all()
    kept = idx >= 0
    assert (r16[kept] == (raw[kept].astype(np.float32) / np.float32(meta["div"])).astype(np.float16)).all()
    assert (r16[~kept].view(np.uint16) == 0xFBFF).all()


FUSED = np.load(Path(__file__).resolve().parent / "golden" / "golden_fused.npz")


def _fused_cases():
    words = ivf.pack_mask_high_first(FUSED["mask"])
    return {"scaled": dict(per_embedding_scale=FUSED["scale"]),
            "scaled_div": dict(per_embedding_scale=FUSED["scale"], divisor_for_int8=16),
            "index_i32": dict(filtering_bit_mask=words, filtering_bit_index=FUSED["mask_index"]),
            "index_scaled": dict(filtering_bit_mask=words, filtering_bit_index=FUSED["mask_index"],
                                 per_embedding_scale=FUSED["scale"], invalid_index_value=-5)}


@pytest.mark.parametrize("name", ["scaled", "scaled_div", "index_i32", "index_scaled"])
def test_fused_kmean_ann_scale_and_mask_rows_match_reference(name):
    """``per_embedding_scale`` (which wins over the divisor) and ``filtering_bit_index`` against
    the reference's CPU scorer (tests/golden/make_golden_fused.py): per row the same (position,
    raw bits) multiset, dtype and pads; the fixture's dots are below 2048, where the CPU and
    CUDA orders of the scaled division agree."""
    kw = _fused_cases()[name]
    raw, idx = ivf.fused_kmean_ann(FUSED["q"], FUSED["offsets"], FUSED["probe"], FUSED["lengths"], FUSED["codes"],
                                   int(FUSED["width"]), **kw)
    want_r, want_i = FUSED[f"{name}_raw"], FUSED[f"{name}_idx"]
    assert raw.dtype == want_r.dtype and raw.shape == want_r.shape
    bits = np.uint16 if raw.dtype == np.float16 else np.int32
    for r in range(raw.shape[0]):
        got, want = idx[r] >= 0, want_i[r] >= 0
        assert sorted(zip(idx[r][got].tolist(), raw[r][got].view(bits).tolist())) == sorted(
            zip(want_i[r][want].tolist(), want_r[r][want].view(bits).tolist()))
        assert (idx[r][~got] == kw.get("invalid_index_value", -1)).all()


@pytest.mark.parametrize("name,fmt", [("f32", "fp32"), ("f16", "fp16")])
def test_fused_kmean_ann_float_rows_match_reference(name, fmt):
    """Float embeddings (entries in {-1, 0, 1}, every partial dot exact) against the reference's
    CPU scorer: the same (position, raw) multiset per row, its pads (-FLT_MAX, -65504) and the
    mask-row index."""
    words = ivf.pack_mask_high_first(FUSED["mask"])
    raw, idx = ivf.fused_kmean_ann(FUSED["tern_q"].astype(np.float32), FUSED["offsets"], FUSED["probe"],
                                   FUSED["lengths"], FUSED["tern_x"].astype(np.float32), int(FUSED["width"]),
                                   filtering_bit_mask=words, filtering_bit_index=FUSED["mask_index"],
                                   invalid_index_value=-2, float_format=fmt)
    want_r, want_i = FUSED[f"{name}_raw"], FUSED[f"{name}_idx"]
    for r in range(raw.shape[0]):
        got, want = idx[r] >= 0, want_i[r] >= 0
        assert sorted(zip(idx[r][got].tolist(), raw[r][got].astype(np.float32).tolist())) == sorted(
            zip(want_i[r][want].tolist(), want_r[r][want].tolist()))
        assert (raw[r][~got].astype(np.float32) == want_r[r][~want]).all() and (idx[r][~got] == -2).all()


def test_float_chains_round_every_step():
    """The CUDA scorer's fp16 chain rounds after every fused multiply-add and keeps even and odd
    elements apart (simple_index_mm.cuh:96-115): 2048 + 1 + 1 ... stays at 2048 in one lane,
    while the odd lane counts up exactly; fp32 carries both."""
    from oracle import fdot

    x = np.zeros(16)
    x[0::2] = [2048, 1, 1, 1, 1, 1, 1, 1]
    x[1::2] = 1
    q = np.ones(16)
    assert fdot.dot(x, q, "fp16") == 2048 + 8  # even lane stuck at 2048, odd lane 8
    assert fdot.dot(x, q, "fp32") == 2048 + 7 + 8
    assert fdot.unit(96, "fp32") == 96 and fdot.unit(256, "fp32") == 64 and fdot.unit(192, "fp16") == 192
    assert fdot.unit(72, "fp32") == 0 and fdot.unit(20, "fp16") == 0


def test_scaled_division_rounds_the_dot_to_fp16_first():
    """The CUDA scorer divides Half(dot) by the Half scale (index_mm_helpers.cuh:49-53); above
    2048 an integer dot is not exact in fp16, so its result differs from the CPU scorer's
    Half(float(dot) / scale) (fused_kmean_ann.cpp:196-199) for some dots: the restatement follows
    the CUDA op it replaces."""
    codes = np.ones((1, 65), dtype=np.int8)
    q = np.full((1, 65), 32, dtype=np.int8)
    q[0, 64] = 1  # dot 2049: fp16 rounds it to 2048
    scale = np.array([3.0], dtype=np.float16)
    raw, _ = ivf.fused_kmean_ann(q, np.array([0, 1]), np.array([[0]]), np.array([[1]]), codes, 32,
                                 per_embedding_scale=scale)
    cuda_form = np.float16(np.float32(np.float16(2049.0)) / np.float32(3.0))  # 682.5
    cpu_form = np.float16(np.float32(2049.0) / np.float32(3.0))  # 683
    assert raw[0, 0] == cuda_form and cuda_form != cpu_form


def test_fused_kmean_ann_mask_and_clipping():
    """A cluster longer than the row fills the row's whole warps; slots whose mask bit is
    clear keep the pads."""
    sizes = np.array([70, 5, 40], dtype=np.int64)
    offsets = np.r_[0, np.cumsum(sizes)]
    rng = np.random.default_rng(3)
    codes = rng.integers(-127, 128, (int(sizes.sum()), 8), dtype=np.int8)
    q = rng.integers(-127, 128, (2, 8), dtype=np.int8)
    probe = np.array([[1, 0, 2], [2, 1, 0]])
    raw, idx = ivf.fused_kmean_ann(q, offsets, probe, sizes[probe], codes, 64)
    # positions: cluster 0 = 0..69, cluster 1 = 70..74, cluster 2 = 75..114
    # row 0: cluster 1 has no whole warp, cluster 0 clipped to 64 fills the row
    assert idx[0].tolist() == list(range(0, 64))
    # row 1: cluster 2's first warp, then the first 32 of cluster 0's clipped 64
    assert idx[1].tolist() == list(range(75, 107)) + list(range(0, 32))
    mask = np.ones((2, int(sizes.sum())), dtype=bool)
    mask[:, 10] = False
    rm, im = ivf.fused_kmean_ann(q, offsets, probe, sizes[probe], codes, 64,
                                 filtering_bit_mask=ivf.pack_mask_high_first(mask))
    assert im[0, 10] == -1 and rm[0, 10] == ivf.INT32_MIN and im[1, 42] == -1 and rm[1, 42] == ivf.INT32_MIN
    im[0, 10], im[1, 42] = idx[0, 10], idx[1, 42]
    rm[0, 10], rm[1, 42] = raw[0, 10], raw[1, 42]
    assert (im == idx).all() and (rm == raw).all()


def test_slot_order_is_warp_prefixes_then_remainders():
    """Clusters of 33 and 5 items probed as [1, 0], every item tied: the kept ids
    follow the CUDA scorer's slots (cluster 0's first 32, then the remainders in
    probe order: cluster 1's five, cluster 0's 33rd), not the probe-order
    concatenation."""
    sizes = np.array([33, 5, 7], dtype=np.int64)
    offsets = np.r_[0, np.cumsum(sizes)]
    order = ivf.probe_slots(np.array([1, 0]), offsets, sizes)
    assert order.tolist() == list(range(0, 32)) + list(range(33, 38)) + [32]
    other = ivf.probe_slots(np.array([0, 1]), offsets, sizes)
    assert other.tolist() == list(range(0, 32)) + [32] + list(range(33, 38))
    codes = np.ones((int(offsets[-1]), 8), dtype=np.int8)
    q = np.ones((1, 8), dtype=np.float32)
    sort_perm = np.arange(int(offsets[-1]))[::-1].copy()
    ids, scores = ivf.search(q, np.array([[1, 0]]), offsets, sizes, codes, sort_perm, np.float32(0.5), 40, 38)
    assert (ids[0, :38] == sort_perm[order]).all() and (ids[0, 38:] == -1).all()
    assert np.isneginf(scores[0, 38:]).all() and (scores[0, :38] == scores[0, 0]).all()


def test_k_above_width_pads():
    sizes = np.array([3], dtype=np.int64)
    offsets = np.array([0, 3])
    codes = np.array([[1, 0], [0, 1], [2, 2]], dtype=np.int8)
    ids, scores = ivf.search(np.array([[1.0, 0.5]], np.float32), np.array([[0]]), offsets, sizes, codes,
                             np.array([10, 11, 12]), np.float32(1.0), 40, 3)
    # width rounds up to 32 slots; only the 3 written ones are returned
    assert ids[0, :3].tolist() == [12, 10, 11] and (ids[0, 3:] == -1).all()
    assert np.isneginf(scores[0, 3:]).all()


def test_row_wider_than_width_is_rejected():
    sizes = np.array([40], dtype=np.int64)
    with pytest.raises(ValueError):
        ivf.search(np.ones((1, 4), np.float32), np.array([[0]]), np.array([0, 40]), sizes,
                   np.ones((40, 4), np.int8), np.arange(40), np.float32(1.0), 5, 32)


def test_probe_prep_cumsums():
    """st::probe_prep's outputs as the reference checks them
    (retrieve/tests/parity/test_official.py:676-697)."""
    rng = np.random.default_rng(9)
    sizes = rng.integers(0, 150, 300)
    offsets = np.r_[0, np.cumsum(sizes)]
    probe = np.argsort(rng.random((20, 300)), axis=1)[:, :24]
    q = rng.standard_normal((20, 128)).astype(np.float32)
    out = ivf.probe_prep(q, probe, offsets, sizes)
    codes, scales = knn.quantize_int8(q)
    assert np.array_equal(out[0], codes) and np.array_equal(out[1], scales)
    length = sizes[probe]
    assert np.array_equal(out[3], length) and np.array_equal(out[4], offsets[probe])
    warps = (length // 32).reshape(-1)
    assert np.array_equal(out[5], warps)
    assert np.array_equal(out[6], np.cumsum((warps * 32).reshape(probe.shape), axis=1))
    assert np.array_equal(out[7], np.cumsum((length % 32).reshape(-1)))
    assert np.array_equal(out[8], np.cumsum(warps))
    # the slot order's split point per row is the row's last warp-rounded cumsum
    for r in range(3):
        pos = ivf.probe_slots(probe[r], offsets, sizes)
        assert len(pos) == int(length[r].sum())
        cluster = np.searchsorted(offsets, pos, side="right") - 1
        in_warp_prefix = (pos - offsets[cluster]) < sizes[cluster] // 32 * 32
        head = int(out[6][r, -1])
        assert in_warp_prefix[:head].all() and not in_warp_prefix[head:].any()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_exact_layout_and_test_equal_the_clause_predicate(seed):
    """The exact filter's layout (adapter.py:68-89) and test (fork_filters.cuh:15-41) give
    the LiNR clause predicate (pinned to the reference by golden.npz): the reference's own
    gate feeds both the same predicate (retrieve/tests/parity/test_official.py:278-293)."""
    from oracle import filters

    rng = np.random.default_rng(seed)
    n, c, a = 700, 4, 3
    attrs = rng.integers(-1, 6, (n, c, a))
    attrs[rng.random(n) < 0.1, 2, :] = -1  # docs with no value in a clause
    rev = rng.random(c) < 0.5
    q = rng.integers(-1, 6, (9, c))
    q[0, 1] = 2**40  # a value no doc can hold: matches nothing
    slots, clause_slots = ivf.exact_layout(attrs)
    assert slots.dtype == np.int32 and slots.shape[1] == n and clause_slots[-1] == slots.shape[0]
    qq = ivf.exact_query(q)
    assert qq[0, 1] == ivf.INT32_MIN
    want = filters.clause_mask(attrs, rev, q)
    for b in range(q.shape[0]):
        assert np.array_equal(ivf.exact_pass(slots, clause_slots, rev, qq[b], np.arange(n)), want[b])


BLOOM = np.load(Path(__file__).resolve().parent / "golden" / "golden_bloom_st.npz")


def test_bloom_plans_match_reference_search():
    """SilverTorch's bloom: its own index build, parser and CPU search ran into the
    fixture (tests/golden/make_golden_bloom_st.py); the restatement of the plan encoding
    and the column-word evaluation gives the same mask for every plan (nested AND / OR /
    NOT, the empty query, several bundles)."""
    n = int(BLOOM["n"])
    want = np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n].astype(bool)
    assert len(BLOOM["bundle_b_offsets"]) > 2
    for p in range(want.shape[0]):
        got = ivf.bloom_plan_mask(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], BLOOM["plan_data"],
                                  BLOOM["plan_offsets"], p, int(BLOOM["k"]), int(BLOOM["hash_k"]), n)
        assert np.array_equal(got, want[p]), p
    assert want[5].all()  # the empty query matches every doc


def test_bloom_is_a_superset_of_the_exact_predicate():
    """No false negatives (retrieve/tests/parity/test_official.py:455-470) for the plain
    conjunction plans: "0:3" and "0:3 AND 1:5" against the exact clause test."""
    from oracle import filters

    n = int(BLOOM["n"])
    bloom = np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n].astype(bool)
    attrs = BLOOM["attrs"]
    q = np.array([[3, -1, -1], [3, 5, -1]])
    exact = filters.clause_mask(attrs, np.zeros(3, dtype=bool), q)
    assert not (exact & ~bloom[:2]).any()


def test_plan_blob_layout():
    """The prepared blob (adapter.py:212-236): the parser's eight offsets a plan, then its
    data after 8 * slots header words; decoding through the blob gives the same plan."""
    data, offsets = BLOOM["plan_data"], BLOOM["plan_offsets"]
    n_plans = len(offsets) // 8
    blob = ivf.plan_blob(data, offsets, n_plans + 3)
    assert np.array_equal(blob[: len(offsets)], offsets)
    body = blob[8 * (n_plans + 3):].view(np.uint8)[: len(data)]
    assert np.array_equal(body, np.asarray(data).view(np.uint8))
    for p in range(n_plans):
        a = ivf.decode_plan(data, offsets, p)
        b = ivf.decode_plan(body, blob[: 8 * n_plans], p)
        assert all(np.array_equal(x, y) for x, y in zip(a, b, strict=True))


def test_bloom_index_build_matches_reference():
    """The restated builder and feature layout give the reference's own CPU-built index and
    bundle offsets bit for bit (tests/golden/make_golden_bloom_st.py)."""
    fid, off, val = ivf.attrs_to_features(BLOOM["attrs"])
    index, boff = ivf.bloom_index_build(fid, off, val, 10.0, int(BLOOM["k"]))
    assert np.array_equal(boff, BLOOM["bundle_b_offsets"])
    assert np.array_equal(index, BLOOM["bloom_index"])
