"""Pins the CPU oracle (oracle/) to the reference: its outputs against the
golden fixtures made by running the reference's own torch path
(tests/golden/make_golden.py), plus the known-answer facts of the reference's
test suite. CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import bits, dense, filters, knn
from tests.golden import golden_inputs as gi

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")


def _same_topk_up_to_ties(ids, scores, ref_ids, ref_scores, atol):
    """Scores slot-wise within atol; ids equal as sets except for ties at the
    row's last (boundary) score, where torch.topk's choice among equal items is
    unspecified (retrieve/tests/parity/conftest.py:57-98)."""
    assert ids.shape == ref_ids.shape
    np.testing.assert_allclose(scores, ref_scores, atol=atol, rtol=0)
    for r in range(ids.shape[0]):
        fin = np.isfinite(ref_scores[r])
        if not fin.any():
            continue
        last = ref_scores[r][fin].min()
        strict_ref = set(ref_ids[r][fin & (ref_scores[r] > last + atol)].tolist())
        strict_ours = set(ids[r][np.isfinite(scores[r]) & (scores[r] > last + atol)].tolist())
        assert strict_ref == strict_ours, f"row {r}: ids above the boundary score differ"


def test_c1_fullscan_matches_reference():
    q, x = gi.c1_inputs()
    ids, scores = dense.dense_topk(q, x, 10)
    _same_topk_up_to_ties(ids, scores, GOLDEN["c1_ids"], GOLDEN["c1_scores"], atol=1e-6)


def test_clause_filter_matches_reference():
    attrs, rev, qa = gi.clause_inputs()
    m = filters.clause_mask(attrs.numpy(), rev.numpy(), qa.numpy())
    ref = np.unpackbits(GOLDEN["clause_mask"], axis=1)[:, : attrs.shape[0]].astype(bool)
    assert np.array_equal(m, ref)
    import torch

    sc = torch.randn(qa.shape[0], attrs.shape[0], generator=torch.Generator().manual_seed(4)).numpy()
    assert np.array_equal(filters.clause_mask_scores(sc, attrs.numpy(), rev.numpy(), qa.numpy()),
                          GOLDEN["clause_mask_scores"])
    ids, counts = filters.clause_compact(attrs.numpy(), rev.numpy(), qa.numpy())
    assert np.array_equal(counts, GOLDEN["clause_counts"])
    assert np.array_equal(ids, GOLDEN["clause_ids_head"])


def test_fused_masked_knn_topk_matches_reference():
    q, x, pos, counts = gi.fmkt_inputs()
    ids, scores = knn.fused_masked_knn_topk(q, x, pos, counts, 20)
    _same_topk_up_to_ties(ids, scores, GOLDEN["fmkt_ids"], GOLDEN["fmkt_scores"], atol=1e-5)
    assert (ids[1, 7:] == -1).all() and np.isneginf(scores[1, 7:]).all()


def test_oporp_matches_reference():
    qb, xb, pos, counts = gi.oporp_inputs()
    ids, scores = knn.oporp_full(qb.numpy(), xb.numpy(), 50)
    _same_topk_up_to_ties(ids, scores, GOLDEN["oporp_full_ids"], GOLDEN["oporp_full_scores"], atol=0)
    ids, scores = knn.oporp_indirect(qb.numpy(), xb.numpy(), 50, pos.numpy(), counts.numpy())
    _same_topk_up_to_ties(ids, scores, GOLDEN["oporp_ind_ids"], GOLDEN["oporp_ind_scores"], atol=0)


def test_quantize_int8_matches_reference():
    """The fixture was made by the reference's ``quantize_int8`` on CPU tensors, where
    torch divides by 127; on CUDA tensors (the path this package replaces) torch and
    SilverTorch's prep multiply by fp32(1/127). Codes agree in both; the CPU scales
    are pinned exactly, and the device scales sit within one ulp of them."""
    x = gi.quantize_inputs().numpy()
    codes, cpu_scales = knn.quantize_int8(x, device_scale=False)
    assert np.array_equal(codes, GOLDEN["q8_codes"])
    assert np.array_equal(cpu_scales, GOLDEN["q8_scales"])
    dev_codes, dev_scales = knn.quantize_int8(x)
    assert np.array_equal(dev_codes, codes)
    gap = np.abs(dev_scales.view(np.int32).astype(np.int64) - cpu_scales.view(np.int32).astype(np.int64))
    assert gap.max() <= 1
    abs_max = np.maximum(np.abs(x).max(axis=1), np.float32(1e-8))
    recip = np.float32(1.0) / np.float32(127.0)
    assert np.array_equal(dev_scales, (abs_max * recip).astype(np.float32))


def test_quantize_int8_device_edge_rows():
    """The rows ``st::probe_prep`` is checked on against ``quantize_int8``
    (retrieve/tests/parity/test_official.py:676-697): all zeros, one tiny value, and
    quotients that land exactly on a half code (ties round to even)."""
    d = 16
    x = np.zeros((3, d), dtype=np.float32)
    x[1, 3] = np.float32(1e-30)
    x[2] = (np.arange(d) % 3 - 1.0).astype(np.float32)
    x[2, 0] = np.float32(2.54)
    x[2, 1:5] = np.array([0.01, -0.01, 1.27, -1.27], dtype=np.float32)
    codes, scales = knn.quantize_int8(x)
    assert (codes[0] == 0).all() and scales[0] == np.float32(1e-8) * (np.float32(1) / np.float32(127))
    assert (codes[1] == 0).all()  # 1e-30 is below the 1e-8 floor of abs_max
    # 127 * x / 2.54 for x = ±0.01, ±1.27 is ±0.5, ±63.5 up to the fp32 rounding of the quotient
    ratio = (x[2].astype(np.float64) / np.float64(np.float32(2.54))).astype(np.float32)
    want = np.clip(np.rint(ratio * np.float32(127.0)), -128, 127).astype(np.int8)
    assert np.array_equal(codes[2], want)
    assert codes[2, 0] == 127


def test_quantize_int8_known_constants():
    """retrieve/tests/correctness/test_quantize.py:100-130."""
    x = np.array([[1.0, -1.0, 0.5, -0.25, 1e-8, 0.0, 0.7, -0.7],
                  [2.0, -2.0, 1.0, -0.5, 1e-8, 0.0, 1.4, -1.4]], dtype=np.float32)
    codes, scales = knn.quantize_int8(x)
    assert codes[0, 0] == 127 and codes[0, 1] == -127 and codes[1, 0] == 127 and codes[1, 1] == -127
    assert codes.max() <= 127 and codes.min() >= -127
    np.testing.assert_allclose(scales, np.array([1.0, 2.0]) / 127.0, atol=1e-6)
    z_codes, z_scales = knn.quantize_int8(np.zeros((4, 8), dtype=np.float32))
    assert (z_codes == 0).all() and np.isfinite(z_scales).all()


def test_sign_packing_matches_reference_simhash():
    xs = gi.simhash_inputs().numpy()
    proj = xs @ GOLDEN["simhash_R"].T
    assert np.array_equal(bits.pack_signs(proj), GOLDEN["simhash_bits"])


def test_popcount_matches_reference_and_known_constants():
    assert np.array_equal(bits.popcount(GOLDEN["popcount_in"]), GOLDEN["popcount_out"])
    got = bits.popcount(np.array([0, 1, 2, 3, -1, 0x5555555555555555], dtype=np.int64))
    assert got.tolist() == [0, 1, 1, 2, 64, 32]  # retrieve/tests/correctness/test_quantize.py:195-199


@pytest.mark.parametrize("seed", [0, 1])
def test_popcount_against_python_bin(seed):
    rng = np.random.default_rng(seed)
    x = rng.integers(np.iinfo(np.int64).min, np.iinfo(np.int64).max, size=64, dtype=np.int64)
    exp = [bin(int(v) & 0xFFFFFFFFFFFFFFFF).count("1") for v in x]
    assert bits.popcount(x).tolist() == exp


def test_gemv_oracle_is_sequential_fma():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 128)).astype(np.float16)
    et = rng.standard_normal((128, 40)).astype(np.float16)
    out = knn.gemv_scores(q, et)
    acc = np.zeros(40, dtype=np.float64)
    for k in range(128):  # fp64 emulation of fp32 FMA: exact product, one rounding per step
        acc = (q[0, k].astype(np.float64) * et[k].astype(np.float64) + acc).astype(np.float32).astype(np.float64)
    np.testing.assert_array_equal(out[0], acc.astype(np.float32))


GOLDEN_INT8 = np.load(Path(__file__).resolve().parent / "golden" / "golden_int8.npz")


@pytest.mark.parametrize("d", [128, 256])
def test_int8_raw_dots_match_reference_fused_kmean_ann(d):
    # raw int32 dots of SilverTorch's CPU scorer (tests/golden/make_golden_int8.py)
    q = GOLDEN_INT8[f"queries_{d}"].astype(np.int64)
    x = GOLDEN_INT8[f"items_{d}"].astype(np.int64)
    dots = q @ x.T
    assert np.array_equal(dots.astype(np.int32), GOLDEN_INT8[f"dots_{d}"])
    # the oracle's dequant with unit scales is the raw dot as fp32 (|dot| < 2^24)
    ids, scores = knn.silvertorch_fullprobe_codes(GOLDEN_INT8[f"queries_{d}"], GOLDEN_INT8[f"items_{d}"], 1.0, 1.0, 50)
    top = np.sort(GOLDEN_INT8[f"dots_{d}"], axis=1)[:, ::-1][:, :50].astype(np.float32)
    assert np.array_equal(scores, top)


QUANT = np.load(Path(__file__).resolve().parent / "golden" / "golden_quant.npz")


def _ulp_gap(a, b):
    return int(np.abs(np.float32(a).view(np.int32).astype(np.int64) - np.float32(b).view(np.int32).astype(np.int64)))


def test_quantize_int8_global_matches_reference():
    """tests/golden/make_golden_quant.py ran the reference's quantize_int8_global on CPU
    tensors (scale = abs_max / 127); the device form multiplies by fp32(1/127)."""
    for rows, codes_key, scale_key in ((None, "global_codes", "global_scale"),
                                       (QUANT["global_perm"], "global_codes_perm", "global_scale_perm")):
        codes, cpu_scale = knn.quantize_int8_global(QUANT["global_x"], rows=rows, device_scale=False)
        assert np.array_equal(codes, QUANT[codes_key])
        assert np.float32(cpu_scale) == QUANT[scale_key]
        dev_codes, dev_scale = knn.quantize_int8_global(QUANT["global_x"], rows=rows)
        assert np.array_equal(dev_codes, codes) and _ulp_gap(dev_scale, cpu_scale) <= 1
    codes, scale = knn.quantize_int8_global(QUANT["global_nan_x"], device_scale=False)
    assert np.array_equal(codes, QUANT["global_nan_codes"]) and np.isnan(scale) and np.isnan(QUANT["global_nan_scale"])


def test_quantize_int8_nan_and_inf_rows_match_reference():
    codes, scales = knn.quantize_int8(QUANT["q8_special_x"], device_scale=False)
    assert np.array_equal(codes, QUANT["q8_special_codes"])
    assert np.array_equal(scales, QUANT["q8_special_scales"], equal_nan=True)
    assert np.isnan(scales[1]) and (codes[1] == 0).all() and np.isinf(scales[2])


def test_sign_packing_matches_reference_edge_values():
    """Zeros, negative zeros, NaN (all 0 bits) and the smallest subnormals (signed)."""
    assert np.array_equal(bits.pack_signs(QUANT["pack_values"]), QUANT["pack_words"])


def test_simhash_and_oporp_packing_match_reference():
    """The reference's own projections (recomputed with torch on CPU, the same calls) packed
    by the oracle equal the reference's codes; pins the bit order of both 1-bit builds."""
    import torch

    embs = torch.from_numpy(QUANT["sim_embs"])
    query = torch.from_numpy(QUANT["sim_query"])
    r = torch.from_numpy(QUANT["sim_r"])
    assert np.array_equal(bits.pack_signs((embs @ r.t()).numpy()), QUANT["sim_bits"])
    assert np.array_equal(bits.pack_signs((query @ r.t()).numpy()), QUANT["sim_qbits"])
    signs = torch.from_numpy(QUANT["oporp_signs"]).to(torch.float32)
    perm = torch.from_numpy(QUANT["oporp_perm"])
    for x, want in ((embs, QUANT["oporp_bits"]), (query, QUANT["oporp_qbits"])):
        proj = (x * signs).index_select(1, perm)  # k_bits = D: one coordinate a bin
        assert np.array_equal(bits.pack_signs(proj.numpy()), want)
