"""Seeded input generators and top-k assertions shared by the parity tests.

Generators follow the reference's fixtures (retrieve/tests/conftest.py:65-133):
N(0, 1) rows, unit-normalised, from a seeded torch CPU generator (so the same
seed gives the same tensors on every machine), then moved to the device.
"""

from __future__ import annotations

import numpy as np
import torch


def make_rows(n: int, d: int, *, seed: int, dtype=torch.float32, normalized=True, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g)
    if normalized:
        x = x / x.norm(dim=1, keepdim=True).clamp_min(1e-8)
    return x.to(dtype).to(device)


def make_int_rows(n: int, d: int, *, seed: int, lo=-3, hi=4, dtype=torch.bfloat16, device="cpu"):
    """Small-integer rows: every dot product is an exact fp32 integer whatever
    the accumulation order, so tensor-core scores are bit-comparable to the
    oracle and ties are plentiful."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(lo, hi, (n, d), generator=g).to(torch.float32)
    return x.to(dtype).to(device)


def mixture_rows(n: int, d: int, *, n_centres: int, sigma: float, seed: int, dtype, device="cpu", centres=None):
    """The BASELINE corpus family: a Gaussian mixture (centres N(0,1), within
    cluster N(0, sigma^2)), L2-normalised rows."""
    g = torch.Generator().manual_seed(seed)
    if centres is None:
        centres = torch.randn(n_centres, d, generator=g)
    c = torch.randint(0, centres.shape[0], (n,), generator=g)
    x = centres[c] + sigma * torch.randn(n, d, generator=g)
    x = x / x.norm(dim=1, keepdim=True).clamp_min(1e-8)
    return x.to(dtype).to(device), centres


def assert_topk_exact(ids, scores, ref_ids, ref_scores):
    """Bit-exact gate with the strict tie rule: scores equal slot by slot and ids
    equal slot by slot (ties already broken toward the lower id on both sides)."""
    ids = np.asarray(ids)
    scores = np.asarray(scores, dtype=np.float32)
    assert ids.shape == ref_ids.shape, (ids.shape, ref_ids.shape)
    bad_s = ~((scores == ref_scores) | (np.isnan(scores) & np.isnan(ref_scores)))
    assert not bad_s.any(), f"{int(bad_s.sum())} score slots differ; first {np.argwhere(bad_s)[:5].tolist()}"
    bad_i = ids != ref_ids
    assert not bad_i.any(), f"{int(bad_i.sum())} id slots differ; first {np.argwhere(bad_i)[:5].tolist()}"


def assert_topk_close(ids, scores, ref_ids, ref_scores, *, rtol: float, atol: float, min_recall: float):
    """Floating-point gate: sorted scores within atol + rtol*|ref|, and recall of
    the reference id set >= min_recall (boundary near-ties may swap)."""
    ids = np.asarray(ids)
    scores = np.asarray(scores, dtype=np.float32)
    assert ids.shape == ref_ids.shape
    fin = np.isfinite(ref_scores)
    assert np.array_equal(np.isfinite(scores), fin), "non-finite pattern differs"
    err = np.abs(scores[fin] - ref_scores[fin])
    lim = atol + rtol * np.abs(ref_scores[fin])
    assert (err <= lim).all(), f"max score error {err.max()} (limit {lim[err.argmax()]})"
    assert np.all(np.diff(scores, axis=1)[:, :][np.isfinite(scores[:, 1:])] <= 0), "scores not sorted descending"
    tot = hit = 0
    for a, r in zip(ids, ref_ids):
        rs = set(int(v) for v in r if v >= 0)
        tot += len(rs)
        hit += len(rs & set(int(v) for v in a if v >= 0))
    recall = hit / max(tot, 1)
    assert recall >= min_recall, f"recall {recall} < {min_recall}"


def assert_topk_equal_up_to_ties(ids, scores, ref_ids, ref_scores):
    """Scores equal slot by slot (bit for bit); ids equal within every run of
    equal scores as a set, except the row's last run, which may hold any of the
    tied items (two valid tie orders pick different ones at the boundary)."""
    ids = np.asarray(ids)
    scores = np.asarray(scores, dtype=np.float32)
    assert ids.shape == ref_ids.shape
    assert np.array_equal(scores, ref_scores), "scores differ"
    for r in range(ids.shape[0]):
        s = ref_scores[r]
        starts = np.flatnonzero(np.r_[True, s[1:] != s[:-1]])
        ends = np.r_[starts[1:], len(s)]
        for a, b in zip(starts[:-1], ends[:-1]):
            assert set(ids[r, a:b].tolist()) == set(ref_ids[r, a:b].tolist()), f"row {r}: ids differ in slots {a}:{b}"
