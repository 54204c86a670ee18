"""Bit packing and popcount restated in numpy (test infrastructure).

``pack_signs``: retrieve/src/retrieve/indexing/quantize.py:63-72
(``_pack_signs_to_int64``) — bit b of word w is set iff v[64 w + b] > 0.
``popcount``: functional.py:158-170 (``popcount_int64``), exact.
"""

from __future__ import annotations

import numpy as np


def pack_signs(values: np.ndarray) -> np.ndarray:
    v = np.asarray(values)
    *prefix, d = v.shape
    w = d // 64
    bits = (v > 0).reshape(*prefix, w, 64).astype(np.uint64)
    shifts = np.arange(64, dtype=np.uint64)
    words = (bits << shifts).sum(axis=-1, dtype=np.uint64)
    return words.view(np.int64)


def popcount(x: np.ndarray) -> np.ndarray:
    return np.bitwise_count(np.asarray(x, dtype=np.int64).view(np.uint64)).astype(np.int32)
