"""Exact top-k selection with the strict tie rule: score descending, then item id
ascending — the merge rule of the reference's chunked oracle
(evaluation/bench/oracle.py:83-92, ``_merge_topk``: a stable sort by id, then a
stable sort by descending score) and of ``st::search``'s select
(silvertorch/silvertorch/ops/csrc/fork_search_cuda.cu:47-55).

Sentinel semantics follow ``masked_topk`` (retrieve/src/retrieve/functional.py:57-85):
invalid lanes score ``-inf``; with ``sentinel=True`` every winner with a
non-finite score gets id ``-1``; ``pad_to_k`` pads rows with ``-1`` / ``-inf``.
NaN scores rank above everything, as in ``torch.topk``.
"""

from __future__ import annotations

import numpy as np


def _row_order(scores: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """Indices of ``scores`` sorted by (score desc, id asc); NaN first."""
    s = scores.astype(np.float64)
    nan = np.isnan(s)
    s = np.where(nan, np.inf, s)
    # lexsort: last key is primary
    return np.lexsort((ids, ~nan, -s))


def topk_strict(
    scores: np.ndarray,
    k: int,
    *,
    ids: np.ndarray | None = None,
    valid: np.ndarray | None = None,
    pad_to_k: bool = True,
    sentinel: bool = False,
) -> tuple[np.ndarray, np.ndarray]:
    """``[B, P]`` scores → ``(ids [B, k'] int64, scores [B, k'] float32)``.

    ``ids`` maps lanes to item ids (default: lane index); ``valid`` masks lanes
    to ``-inf`` first. ``k' = k`` when ``pad_to_k`` else ``min(k, P)``."""
    scores = np.asarray(scores, dtype=np.float32)
    b, p = scores.shape
    if ids is None:
        ids = np.broadcast_to(np.arange(p, dtype=np.int64), (b, p))
    ids = np.asarray(ids, dtype=np.int64)
    if valid is not None:
        scores = np.where(valid, scores, np.float32(-np.inf))
    kk = min(k, p)
    out_i = np.full((b, k if pad_to_k else kk), -1, dtype=np.int64)
    out_s = np.full((b, k if pad_to_k else kk), -np.inf, dtype=np.float32)
    for r in range(b):
        row_s, row_i = scores[r], ids[r]
        if p > 4 * kk + 64:
            # shortlist: everything >= the kk-th largest value (ties included)
            finite = np.where(np.isnan(row_s), np.inf, row_s)
            kth = np.partition(finite, p - kk)[p - kk]
            cand = np.flatnonzero(finite >= kth)
        else:
            cand = np.arange(p)
        order = cand[_row_order(row_s[cand], row_i[cand])][:kk]
        out_s[r, :kk] = row_s[order]
        out_i[r, :kk] = row_i[order]
    if sentinel:
        out_i = np.where(np.isfinite(out_s), out_i, -1)
    return out_i, out_s


def merge_topk(parts_ids: list[np.ndarray], parts_scores: list[np.ndarray], k: int) -> tuple[np.ndarray, np.ndarray]:
    """Top-k of several ``[B, k_i]`` candidate lists (id ``-1`` = empty slot),
    equal scores to the lowest id (evaluation/bench/oracle.py:83-92)."""
    ids = np.concatenate(parts_ids, axis=1)
    sc = np.concatenate(parts_scores, axis=1).astype(np.float32)
    valid = ids >= 0
    return topk_strict(sc, k, ids=np.where(valid, ids, np.iinfo(np.int64).max), valid=valid, sentinel=True)


def is_topk(scores, ks, largest=True):
    """``st::is_topk`` as SilverTorch's CUDA op computes it (silvertorch/ops/csrc/is_topk_cuda.cu
    :63-72, 83-149): per row the value at position ``clamp(k - 1, 0, n - 1)`` of the row sorted
    descending (ascending when not ``largest``), NaN sorting as the largest value, then every
    score ``>=`` (``<=``) it, compared in fp32, flagged 1. Returns float32 0 / 1 flags."""
    s = np.asarray(scores, dtype=np.float32)
    b, n = s.shape
    out = np.zeros((b, n), dtype=np.float32)
    if n == 0:
        return out
    for r in range(b):
        asc = np.sort(s[r])  # NaN last: the largest
        kk = min(max(int(ks[r]) - 1, 0), n - 1)
        kth = asc[::-1][kk] if largest else asc[kk]
        with np.errstate(invalid="ignore"):
            out[r] = (s[r] >= kth) if largest else (s[r] <= kth)
    return out


def take_top_k_and_gather(main_scores, fresh_scores, main_indices, fresh_indices, k, main_data, fresh_data):
    """``st::take_top_k_and_gather_from_main_and_fresh`` (silvertorch/ops/csrc/
    fresh_index_post_processing.cpp:33-128, 226-272) for one data key: the top ``min(k, Mf + Mm)``
    of ``[fresh | main]`` per row, largest first with NaN the largest and ties to the lower merged
    column (the reference's ``torch.topk`` leaves them open), whether each comes from fresh, and
    the winners' data rows (``fresh_data[fresh_indices[b, j]]`` / ``main_data[main_indices[b, j -
    Mf]]``, row 0 for an index outside the table)."""
    main_scores = np.asarray(main_scores, dtype=np.float64)
    fresh_scores = np.asarray(fresh_scores, dtype=np.float64)
    b, mm = main_scores.shape
    mf = fresh_scores.shape[1]
    merged = np.concatenate([fresh_scores, main_scores], axis=1)
    kk = max(0, min(int(k), mf + mm))
    cols = np.zeros((b, kk), dtype=np.int64)
    for r in range(b):
        nan = np.isnan(merged[r])
        key = np.where(nan, np.inf, merged[r])
        order = np.lexsort((np.arange(mf + mm), -key, ~nan))  # NaN first, then larger, then lower column
        cols[r] = order[:kk]
    top = np.take_along_axis(merged, cols, axis=1)
    rows = []
    for r in range(b):
        for c in cols[r]:
            if c < mf:
                i, table = int(np.asarray(fresh_indices)[r, c]), np.asarray(fresh_data)
            else:
                i, table = int(np.asarray(main_indices)[r, c - mf]), np.asarray(main_data)
            rows.append(table[i if 0 <= i < table.shape[0] else 0])
    data = np.stack(rows) if rows else np.zeros((0,) + np.asarray(main_data).shape[1:], np.asarray(main_data).dtype)
    return top, cols, cols < mf, data
