"""Candidate-path, 1-bit and quantization oracles (test infrastructure).

* ``fused_masked_knn_topk``: ops/reference/fused_masked_knn_topk.py:9-29 —
  fp32 dots of the candidates ``positive_indices[b, :counts[b]]``, ``-inf``
  past counts, top-k, ids through ``positive_indices``, non-finite winners -1;
  ties toward the lower candidate index.
* ``oporp_full`` / ``oporp_indirect``: ops/reference/oporp_1bit_match_topk.py:9-41
  — ``64*W - 2*popcount(q ^ x)``; the indirect form returns ``min(k, P)``
  columns.
* ``gemv_scores``: ops/triton/gemv_scores.py:19-28 via the C restatement.
* ``quantize_int8`` / ``quantize_int8_global``: indexing/quantize.py:9-18,
  34-52, with the scale as torch evaluates it on a CUDA tensor (a multiply by
  fp32(1/127)).
"""

from __future__ import annotations

import ctypes

import numpy as np

from oracle.dense import as_f32
from oracle.select import topk_strict


def fused_masked_knn_topk(query, items, positive_indices, counts, k):
    q = as_f32(query)
    x = as_f32(items)
    pos = np.asarray(positive_indices, dtype=np.int64)
    cnt = np.asarray(counts, dtype=np.int64)
    b, p = pos.shape
    scores = np.full((b, p), -np.inf, dtype=np.float32)
    for bi in range(b):
        c = int(min(max(cnt[bi], 0), p))
        ids = pos[bi, :c]
        ok = (ids >= 0) & (ids < x.shape[0])
        s = np.full(c, np.nan, dtype=np.float32)
        if ok.any():
            s[ok] = (x[ids[ok]].astype(np.float64) @ q[bi].astype(np.float64)).astype(np.float32)
        scores[bi, :c] = np.where(ok, s, -np.inf)
    lane_ids, top = topk_strict(scores, k)
    out = np.where(lane_ids >= 0, np.take_along_axis(pos, np.maximum(lane_ids, 0), axis=1), -1)
    out = np.where(np.isfinite(top), out, -1)
    return out, top


def _hamming(qbits: np.ndarray, xbits: np.ndarray) -> np.ndarray:
    """[B, W] x [M, W] uint64 → [B, M] popcount of xor."""
    qb = np.asarray(qbits).view(np.uint64)
    xb = np.asarray(xbits).view(np.uint64)
    return np.bitwise_count(qb[:, None, :] ^ xb[None, :, :]).sum(axis=-1).astype(np.int64)


def oporp_full(query_bits, item_bits, k, chunk=1 << 16):
    qb = np.ascontiguousarray(np.asarray(query_bits, dtype=np.int64))
    xb = np.ascontiguousarray(np.asarray(item_bits, dtype=np.int64))
    w = qb.shape[1]
    best_i = np.zeros((qb.shape[0], 0), dtype=np.int64)
    best_s = np.zeros((qb.shape[0], 0), dtype=np.float32)
    for lo in range(0, xb.shape[0], chunk):
        h = _hamming(qb, xb[lo : lo + chunk])
        s = (64 * w - 2 * h).astype(np.float32)
        ci, cs = topk_strict(s, k, pad_to_k=False)
        all_i = np.concatenate([best_i, ci + lo], axis=1)
        all_s = np.concatenate([best_s, cs], axis=1)
        best_i, best_s = topk_strict(all_s, k, ids=all_i, pad_to_k=False)
    return best_i, best_s


def oporp_indirect(query_bits, item_bits, k, positive_indices, counts):
    qb = np.asarray(query_bits, dtype=np.int64)
    xb = np.asarray(item_bits, dtype=np.int64)
    pos = np.asarray(positive_indices, dtype=np.int64)
    cnt = np.asarray(counts, dtype=np.int64)
    b, p = pos.shape
    w = qb.shape[1]
    scores = np.full((b, p), -np.inf, dtype=np.float32)
    for bi in range(b):
        c = int(min(max(cnt[bi], 0), p))
        ids = pos[bi, :c]
        h = _hamming(qb[bi : bi + 1], xb[ids])[0]
        scores[bi, :c] = (64 * w - 2 * h).astype(np.float32)
    lane_ids, top = topk_strict(scores, k, pad_to_k=False)
    out = np.where(lane_ids >= 0, np.take_along_axis(pos, np.maximum(lane_ids, 0), axis=1), -1)
    out = np.where(np.isfinite(top), out, -1)
    return out, top


_CLIB = None


def _clib():
    global _CLIB
    if _CLIB is None:
        from oracle.build_c import build

        _CLIB = ctypes.CDLL(str(build()))
        _CLIB.oracle_gemv.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_void_p]
    return _CLIB


def gemv_scores(query_f16, items_t_f16) -> np.ndarray:
    q = np.ascontiguousarray(np.asarray(query_f16, dtype=np.float16).reshape(-1))
    et = np.ascontiguousarray(np.asarray(items_t_f16, dtype=np.float16))
    d, n = et.shape
    out = np.empty(n, dtype=np.float32)
    _clib().oracle_gemv(q.ctypes.data, et.ctypes.data, d, n, out.ctypes.data)
    return out.reshape(1, n)


def quantize_int8(x, device_scale: bool = True):
    """indexing/quantize.py:9-18 as it evaluates on a CUDA tensor. The scale
    ``abs_max / 127.0`` is then ``abs_max * fp32(1/127)``: torch computes a
    division by a CPU scalar on the device as a multiply by its fp32
    reciprocal, and SilverTorch's query prep writes the same product
    (silvertorch/ops/csrc/fork_search_cuda.cu:686), which the reference checks
    equal to ``quantize_int8`` on CUDA (retrieve/tests/parity/test_official.py:676-697).
    ``device_scale=False`` gives the CPU evaluation (a correctly rounded
    division), which is what the CPU-generated golden fixture holds. Codes are
    the same either way: the fp64 quotient rounded to fp32, times 127, rounded
    half to even, clamped."""
    x = np.asarray(x, dtype=np.float32)
    abs_max = np.maximum(np.abs(x).max(axis=1, keepdims=True), np.float32(1e-8)).astype(np.float32)
    if device_scale:
        scales = (abs_max * (np.float32(1.0) / np.float32(127.0))).astype(np.float32)[:, 0]
    else:
        scales = (abs_max / np.float32(127.0)).astype(np.float32)[:, 0]
    with np.errstate(invalid="ignore"):
        ratio = (x.astype(np.float64) / abs_max.astype(np.float64)).astype(np.float32)
        codes = _to_int8(np.clip(np.rint(ratio * np.float32(127.0)), -128, 127))
    return codes, scales


def _to_int8(v):
    """fp32 codes to int8, NaN to 0 (torch's conversion of a NaN to an integer)."""
    return np.where(np.isnan(v), 0, v).astype(np.int8)


def quantize_int8_global(x, rows=None, device_scale: bool = True):
    """indexing/quantize.py:34-52: one scale for the whole table.
    ``abs_max = max(max |x|, 1e-8)`` (NaN propagates), codes
    ``clamp(round_half_even(fp32(x / abs_max) * 127), -128, 127)`` for the rows
    ``rows`` (all rows when None), scale ``abs_max * fp32(1/127)`` as on a CUDA
    tensor (``device_scale=False``: the CPU division ``abs_max / 127``). Returns
    ``(codes [n, D] int8, scale float)``."""
    x = np.asarray(x, dtype=np.float32)
    am = np.float32(np.abs(x).max()) if x.size else np.float32(0.0)
    am = np.maximum(am, np.float32(1e-8))
    src = x if rows is None else x[np.asarray(rows, dtype=np.int64)]
    with np.errstate(invalid="ignore", divide="ignore"):
        codes = _to_int8(np.clip(np.rint((src / am).astype(np.float32) * np.float32(127.0)), -128, 127))
    if device_scale:
        scale = np.float32(am * (np.float32(1.0) / np.float32(127.0)))
    else:
        scale = np.float32(am / np.float32(127.0))
    return codes, float(scale)


def int8_topk(query, item_codes, item_scales, k, *, chunk=1 << 18):
    """Int8 scoring oracle: query quantized by ``quantize_int8``; exact int64
    dots; score = (fp32(dot) * q_scale) * item_scale with fp32 rounding after
    each multiply (ops/official/adapter.py:338-367 order); top-k, ties to the
    lower id."""
    codes, qs = quantize_int8(np.asarray(query, dtype=np.float32))
    xc = np.asarray(item_codes, dtype=np.int8)
    xs = np.asarray(item_scales, dtype=np.float32)
    qc = codes.astype(np.int64)
    best_i = np.zeros((qc.shape[0], 0), dtype=np.int64)
    best_s = np.zeros((qc.shape[0], 0), dtype=np.float32)
    for lo in range(0, xc.shape[0], chunk):
        dots = qc @ xc[lo : lo + chunk].astype(np.int64).T
        s = (dots.astype(np.float32) * qs[:, None]).astype(np.float32) * xs[None, lo : lo + chunk]
        ci, cs = topk_strict(s.astype(np.float32), k, pad_to_k=False)
        all_i = np.concatenate([best_i, ci + lo], axis=1)
        all_s = np.concatenate([best_s, cs], axis=1)
        best_i, best_s = topk_strict(all_s, k, ids=all_i, pad_to_k=False)
    return best_i, best_s


def silvertorch_fullprobe_codes(query_codes, item_codes, q_scales, global_scale, k):
    """SilverTorch's int32 path with every cluster probed, on int8 codes (st::search
    semantics, silvertorch fork_search_cuda.cu:1405-1411 and 585-591): rank on the
    raw int32 dot (silvertorch fused_kmean_ann.cpp:60-70), ties in index order,
    then score = (fp32(dot) * q_scale) * global_scale."""
    dots = np.asarray(query_codes, dtype=np.int64) @ np.asarray(item_codes, dtype=np.int64).T
    ids, _ = topk_strict(dots.astype(np.float64).astype(np.float32) if np.abs(dots).max() < 2**24 else dots, k)
    d = np.take_along_axis(dots, ids, axis=1).astype(np.float32)
    qs = np.broadcast_to(np.asarray(q_scales, dtype=np.float32), (d.shape[0],))
    scores = (d * qs[:, None]).astype(np.float32) * np.float32(global_scale)
    return ids, scores.astype(np.float32)


def silvertorch_fullprobe(query, item_codes, global_scale, k):
    """``silvertorch_fullprobe_codes`` after the reference's query quantization
    (``quantize_int8``, retrieve/src/retrieve/indexing/quantize.py:9-18)."""
    codes, qs = quantize_int8(np.asarray(query, dtype=np.float32))
    return silvertorch_fullprobe_codes(codes, item_codes, qs, global_scale, k)
