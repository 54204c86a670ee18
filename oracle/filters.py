"""Exact clause filter restated in numpy (test oracle).

Predicate (retrieve/src/retrieve/functional.py:173-185 ``clause_subset_match``,
used by ops/reference/clause_mask.py:9-21): item n passes query b iff for every
clause c, q[b, c] == -1 (inactive) or (any_a attrs[n, c, a] == q[b, c]) XOR
reverse[c]. ``clause_compact`` (ops/reference/clause_compact.py:9-16 +
functional.py:88-95 ``compact_mask``): the passing ids of each row in ascending
order, and their count.
"""

from __future__ import annotations

import numpy as np


def clause_mask(attrs: np.ndarray, reverse: np.ndarray, qattrs: np.ndarray) -> np.ndarray:
    attrs = np.asarray(attrs, dtype=np.int64)  # [N, C, A]
    qattrs = np.asarray(qattrs, dtype=np.int64)  # [B, C]
    reverse = np.asarray(reverse, dtype=bool)  # [C]
    b = qattrs.shape[0]
    n = attrs.shape[0]
    out = np.ones((b, n), dtype=bool)
    for c in range(attrs.shape[1]):
        cell = attrs[:, c, :]  # [N, A]
        for bi in range(b):
            qv = qattrs[bi, c]
            if qv == -1:
                continue
            match = (cell == qv).any(axis=1)
            out[bi] &= match ^ reverse[c]
    return out


def clause_mask_scores(scores, attrs, reverse, qattrs) -> np.ndarray:
    m = clause_mask(attrs, reverse, qattrs)
    return np.where(m, np.asarray(scores, dtype=np.float32), np.float32(-np.inf))


def clause_compact(attrs, reverse, qattrs):
    """``(ids [B, N] int64 with each row's passing ids first, counts [B])``; the
    tail is -1 here (the kernel leaves it unwritten)."""
    m = clause_mask(attrs, reverse, qattrs)
    b, n = m.shape
    ids = np.full((b, n), -1, dtype=np.int64)
    counts = m.sum(axis=1).astype(np.int64)
    for bi in range(b):
        sel = np.flatnonzero(m[bi])
        ids[bi, : sel.size] = sel
    return ids, counts
