"""The oracle's selection (oracle/select.py) against a brute-force Python
restatement of the reference harness merge rule (evaluation/bench/oracle.py:83-92:
stable sort by id, then stable sort by descending score)."""

from __future__ import annotations

import numpy as np

from oracle.select import merge_topk, topk_strict


def _brute(scores, k):
    out_i, out_s = [], []
    for row in scores:
        order = sorted(range(len(row)), key=lambda i: (-float(row[i]), i))[:k]
        out_i.append(order + [-1] * (k - len(order)))
        out_s.append([float(row[i]) for i in order] + [-np.inf] * (k - len(order)))
    return np.array(out_i), np.array(out_s, dtype=np.float32)


def test_topk_strict_matches_bruteforce_with_ties():
    rng = np.random.default_rng(0)
    for p, k in [(50, 10), (1000, 100), (7, 10), (5000, 3)]:
        sc = rng.integers(-3, 4, size=(6, p)).astype(np.float32)
        i1, s1 = topk_strict(sc, k)
        i2, s2 = _brute(sc, k)
        assert np.array_equal(i1, i2) and np.array_equal(s1, s2)


def test_merge_topk_equals_global_topk():
    rng = np.random.default_rng(1)
    sc = rng.integers(0, 20, size=(4, 3000)).astype(np.float32)
    ref_i, ref_s = topk_strict(sc, 50)
    parts_i, parts_s = [], []
    for lo in range(0, 3000, 700):
        pi, ps = topk_strict(sc[:, lo : lo + 700], 50, pad_to_k=False)
        parts_i.append(pi + lo)
        parts_s.append(ps)
    mi, ms = merge_topk(parts_i, parts_s, 50)
    assert np.array_equal(mi, ref_i) and np.array_equal(ms, ref_s)


def test_valid_mask_and_sentinel():
    sc = np.array([[3.0, 1.0, 2.0]], dtype=np.float32)
    ids, s = topk_strict(sc, 4, valid=np.array([[True, False, True]]), sentinel=True)
    assert ids.tolist() == [[0, 2, -1, -1]]
    assert s[0, :2].tolist() == [3.0, 2.0] and np.isneginf(s[0, 2:]).all()
