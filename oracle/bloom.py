"""Per-item Bloom filter restated in numpy (test infrastructure).

Hash: MurmurHash3 x64-128 of the 16-byte key (feature id, feature value) with a
64-bit seed, the two halves XOR-ed (silvertorch/silvertorch/ops/csrc/
bloom_index_util.cuh:61-107 ``murmur_hash3_2x64``; Appleby's published
algorithm). Build positions: the first k distinct ``hash(id, value, seed) % b``
for seed = 0, 1, 2, ... (bloom_index_util.cuh:185-208). Search positions: the
first k distinct among the first ``n_stored`` hashes (bloom_index_search_cuda.cu
:304-349 ``signature_match<true>``), so a term may test fewer than k bits.

Layout: one uint64 word per item with bit p set iff position p is set — the
transpose of the reference's bundle rows (``bloom_index[p * 32 + doc // 64]``
bit ``63 - doc % 64`` for a one-bundle, b = 64 index).
"""

from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1


def _rotl(x: int, r: int) -> int:
    return ((x << r) | (x >> (64 - r))) & M64


def murmur_hash3_2x64(x: int, y: int, seed: int) -> int:
    c1, c2 = 0x87C37B91114253D5, 0x4CF5AD432745937F
    x &= M64
    y &= M64
    h1 = h2 = seed & M64
    k1 = (x * c1) & M64
    k1 = _rotl(k1, 31)
    k1 = (k1 * c2) & M64
    h1 ^= k1
    h1 = _rotl(h1, 27)
    h1 = (h1 + h2) & M64
    h1 = (h1 * 5 + 0x52DCE729) & M64
    k2 = (y * c2) & M64
    k2 = _rotl(k2, 33)
    k2 = (k2 * c1) & M64
    h2 ^= k2
    h2 = _rotl(h2, 31)
    h2 = (h2 + h1) & M64
    h2 = (h2 * 5 + 0x38495AB5) & M64
    h1 ^= 16
    h2 ^= 16
    h1 = (h1 + h2) & M64
    h2 = (h2 + h1) & M64
    for name in ("h1", "h2"):
        v = h1 if name == "h1" else h2
        v ^= v >> 33
        v = (v * 0xFF51AFD7ED558CCD) & M64
        v ^= v >> 33
        v = (v * 0xC4CEB9FE1A85EC53) & M64
        v ^= v >> 33
        if name == "h1":
            h1 = v
        else:
            h2 = v
    h1 = (h1 + h2) & M64
    h2 = (h2 + h1) & M64
    return h1 ^ h2


def build_positions(fid: int, value: int, b: int, k: int) -> list[int]:
    out: list[int] = []
    seed = 0
    while len(out) < k:
        p = murmur_hash3_2x64(fid, value, seed) % b
        seed += 1
        if p not in out:
            out.append(p)
    return out


def search_positions(fid: int, value: int, b: int, k: int, n_stored: int) -> list[int]:
    out: list[int] = []
    for seed in range(n_stored):
        if len(out) >= k:
            break
        p = murmur_hash3_2x64(fid, value, seed) % b
        if p not in out:
            out.append(p)
    return out


def term_mask(fid: int, value: int, k: int, n_stored: int, b: int = 64) -> int:
    m = 0
    for p in search_positions(fid, value, b, k, n_stored):
        m |= 1 << p
    return m


def item_words(attrs: np.ndarray, k: int, b: int = 64) -> np.ndarray:
    """[N, C, A] int64 (-1 pad; clause index = feature id) → [N] uint64 words."""
    attrs = np.asarray(attrs, dtype=np.int64)
    if attrs.ndim == 2:
        attrs = attrs[:, :, None]
    cache: dict[tuple[int, int], int] = {}
    out = np.zeros(attrs.shape[0], dtype=np.uint64)
    for n in range(attrs.shape[0]):
        w = 0
        for c in range(attrs.shape[1]):
            for v in attrs[n, c]:
                if v == -1:
                    continue
                key = (c, int(v))
                if key not in cache:
                    m = 0
                    for p in build_positions(c, int(v), b, k):
                        m |= 1 << p
                    cache[key] = m
                w |= cache[key]
        out[n] = np.uint64(w)
    return out


def transpose_reference_bundle(bloom_index: np.ndarray, n_docs: int) -> np.ndarray:
    """Reference one-bundle, b = 64 layout → per-item words."""
    bi = np.asarray(bloom_index, dtype=np.int64).view(np.uint64).reshape(64, 32)
    out = np.zeros(n_docs, dtype=np.uint64)
    for d in range(n_docs):
        col, bit = d // 64, 63 - d % 64
        w = 0
        for p in range(64):
            if (int(bi[p, col]) >> bit) & 1:
                w |= 1 << p
        out[d] = np.uint64(w)
    return out
