"""Dense exact search oracle: ``FullScanKNN`` / ``PostfilterKNN`` semantics.

``FullScanKNN.forward`` (retrieve/src/retrieve/modules/knn.py:153-170) scores
``query @ item_embs.t()`` in the input dtype and takes ``torch.topk``;
``PostfilterKNN.score`` (knn.py:62-69) casts both sides to fp16 and
accumulates in fp32 (``torch.mm(..., out_dtype=float32)``). This restatement
computes fp32 dot products of the (already rounded) inputs chunk by chunk, the
way the reference harness oracle does (evaluation/bench/oracle.py:96-158: item
chunks, query batches, a running top-k merged with ``_merge_topk``), and breaks
ties toward the lower id.
"""

from __future__ import annotations

import numpy as np

from oracle.select import topk_strict


def as_f32(x) -> np.ndarray:
    """A numpy fp32 copy of a torch tensor (any float dtype) or array."""
    try:
        import torch

        if isinstance(x, torch.Tensor):
            return x.detach().to("cpu", torch.float32).numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, dtype=np.float32)


def dense_topk(queries, items, k: int, *, item_chunk: int = 1 << 20, query_batch: int = 256):
    """Exact top-k of ``queries @ items.T`` (fp32) → ``(ids [B, k], scores [B, k])``."""
    q = as_f32(queries)
    x = as_f32(items)
    b, n = q.shape[0], x.shape[0]
    out_i = np.full((b, k), -1, dtype=np.int64)
    out_s = np.full((b, k), -np.inf, dtype=np.float32)
    for qs in range(0, b, query_batch):
        qe = min(b, qs + query_batch)
        best_i = np.full((qe - qs, 0), -1, dtype=np.int64)
        best_s = np.full((qe - qs, 0), -np.inf, dtype=np.float32)
        for cs in range(0, n, item_chunk):
            ce = min(n, cs + item_chunk)
            sc = q[qs:qe] @ x[cs:ce].T
            ci, cv = topk_strict(sc, k, pad_to_k=False)
            ci = ci + cs
            all_i = np.concatenate([best_i, ci], axis=1)
            all_s = np.concatenate([best_s, cv], axis=1)
            best_i, best_s = topk_strict(all_s, k, ids=all_i, pad_to_k=False)
        out_i[qs:qe, : best_i.shape[1]] = best_i
        out_s[qs:qe, : best_s.shape[1]] = best_s
    return out_i, out_s


def recall_at_k(ids: np.ndarray, ref_ids: np.ndarray) -> float:
    """Mean over rows of |ids ∩ ref_ids| / |ref_ids| (ids -1 ignored)."""
    tot, hit = 0, 0
    for a, r in zip(ids, ref_ids):
        rs = set(int(v) for v in r if v >= 0)
        tot += len(rs)
        hit += len(rs & set(int(v) for v in a if v >= 0))
    return hit / max(tot, 1)
