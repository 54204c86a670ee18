"""Quantizers and 1-bit packers on the device, with the names, arguments and
results of ``retrieve.indexing.quantize`` (retrieve/src/retrieve/indexing/quantize.py).

* ``quantize_int8`` (:9-18): the per-row query quantizer, ``ops.quantize_int8``.
* ``quantize_int8_global`` (:34-52): one scale for the table, ``rb_quantize_int8_global``;
  ``rows`` quantizes ``embs[rows]`` (the cluster-sorted build) without the gathered copy.
* ``pack_signs`` (``_pack_signs_to_int64``, :63-72): bit b of word w set iff
  ``values[..., 64 w + b] > 0``, ``rb_pack_signs`` (one warp ballot per 32 values instead
  of an ``[..., W, 64]`` int64 temporary).
* ``quantize_simhash_1bit`` / ``project_simhash_1bit_query`` (:143-172) and
  ``quantize_oporp_1bit`` / ``project_oporp_1bit_query`` (:75-140): the projections are
  the same torch calls the reference makes (its generator draws, its GEMM through
  cuBLAS, its OPORP binning), so on the same device they give the same values; the
  packing is ``pack_signs``.

Scales are the CUDA evaluation of ``abs_max / 127.0`` (``abs_max * fp32(1/127)``).
CUDA tensors only; there is no CPU path.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from retrieve_b200 import _lib, ops

_lib.lib()  # no fallback: a missing library fails the import


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _cuda(*tensors: Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("retrieve_b200.quantize runs on CUDA tensors only")


def quantize_int8(embs: Tensor) -> tuple[Tensor, Tensor]:
    """Per-row symmetric int8: ``(codes [B, D] int8, scales [B] fp32)``."""
    return ops.quantize_int8(embs)


def quantize_int8_global(embs: Tensor, rows: Tensor | None = None) -> tuple[Tensor, float]:
    """Per-tensor symmetric int8 over ``embs`` ``[N, D]`` fp32: ``(codes, scale)`` with
    codes for ``embs[rows]`` (every row when ``rows`` is None)."""
    if embs.dim() != 2:
        raise ValueError(f"expected 2-D [N, D] embeddings, got shape {tuple(embs.shape)}")
    if embs.dtype != torch.float32:
        raise TypeError(f"quantize_int8_global takes float32 embeddings, got {embs.dtype}")
    if embs.numel() == 0:
        raise RuntimeError("quantize_int8_global: empty table (no abs-max to take)")
    _cuda(embs)
    x = embs.contiguous()
    n, d = x.shape
    idx = None
    n_rows = n
    if rows is not None:
        _cuda(rows)
        idx = rows.to(torch.int64).contiguous().view(-1)
        if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= n):
            raise IndexError(f"rows index out of range for {n} rows")
        n_rows = idx.numel()
    codes = torch.empty((n_rows, d), dtype=torch.int8, device=x.device)
    scale = torch.empty((1,), dtype=torch.float32, device=x.device)
    ws = torch.empty(256, dtype=torch.uint8, device=x.device)
    rc = _lib.lib().rb_quantize_int8_global(
        ctypes.c_void_p(x.data_ptr()), n, d, ctypes.c_void_p(0 if idx is None else idx.data_ptr()), n_rows,
        ctypes.c_void_p(codes.data_ptr()), ctypes.c_void_p(scale.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
        ws.numel(), _stream(x.device),
    )
    _lib.check(rc, "quantize_int8_global")
    return codes, float(scale.item())


def pack_signs(values: Tensor) -> Tensor:
    """``[..., 64 W]`` fp32 → ``[..., W]`` int64 sign words (LSB first)."""
    if values.dim() < 1 or values.shape[-1] % 64 != 0:
        raise ValueError(f"the last dimension must be a multiple of 64, got {tuple(values.shape)}")
    _cuda(values)
    *prefix, d = values.shape
    v = values.to(torch.float32).contiguous().view(-1, d)
    out = torch.empty((v.shape[0], d // 64), dtype=torch.int64, device=v.device)
    rc = _lib.lib().rb_pack_signs(ctypes.c_void_p(v.data_ptr()), v.shape[0], d, ctypes.c_void_p(out.data_ptr()),
                                  _stream(v.device))
    _lib.check(rc, "pack_signs")
    return out.view(*prefix, d // 64)


# --- 1-bit codes ------------------------------------------------------------------------------
# A 1-bit code is the sign pattern of a random linear sketch of the embedding, packed by
# ``pack_signs``. The sketches are drawn from a torch generator seeded like the reference's
# builds (the same draws in the same order, on the embeddings' device), so a table and its
# queries built here carry the reference's bits; everything around the draws (blocking,
# packing, validation) is this module's own.

_BLOCK_ROWS = 1 << 16  # table rows sketched per block: bounds the fp32 sketch buffer


def _matrix(x: Tensor, what: str) -> None:
    if x.dim() != 2:
        raise ValueError(f"{what} must be a 2-D [rows, dim] tensor, got shape {tuple(x.shape)}")
    _cuda(x)


def _codes(embs: Tensor, n_bits: int, sketch) -> Tensor:
    """``[N, n_bits // 64]`` int64 sign words of ``sketch(embs)``, one row block at a time."""
    n = embs.shape[0]
    out = torch.empty((n, n_bits // 64), dtype=torch.int64, device=embs.device)
    lo = 0
    while lo < n:
        hi = min(n, lo + _BLOCK_ROWS)
        out[lo:hi] = pack_signs(sketch(embs[lo:hi]))
        lo = hi
    return out


def _gaussian_sketch(d: int, n_bits: int, seed: int, device: torch.device) -> Tensor:
    """SimHash's ``[n_bits, D]`` N(0, 1) projection: one ``randn`` from a generator seeded
    with ``seed`` on ``device`` (indexing/quantize.py:143-145 draws it so)."""
    gen = torch.Generator(device=device).manual_seed(int(seed))
    return torch.randn(n_bits, d, generator=gen, device=device)


def quantize_simhash_1bit(embs: Tensor, k_bits: int, seed: int = 0) -> tuple[Tensor, Tensor]:
    """SimHash codes ``(bits [N, k_bits // 64] int64, r [k_bits, D] fp32)``: bit ``j`` of a
    row is the sign of its dot with row ``j`` of ``r``."""
    _matrix(embs, "embs")
    if k_bits <= 0 or k_bits % 64:
        raise ValueError(f"SimHash codes are packed in 64-bit words: k_bits={k_bits} is not a positive multiple "
                         "of 64")
    r = _gaussian_sketch(embs.shape[1], k_bits, seed, embs.device)
    return _codes(embs, k_bits, lambda rows: rows @ r.t()), r


def project_simhash_1bit_query(query: Tensor, r: Tensor) -> Tensor:
    """A query batch's SimHash code under the table's ``r``: ``[B, k_bits // 64]`` int64."""
    _matrix(query, "query")
    return pack_signs(query @ r.t())


def _oporp_bits(d: int, k_bits: int) -> int:
    """Sign-OPORP's code length: ``k_bits`` (0: one bit per coordinate), which must split the
    ``d`` coordinates into equal bins and fill whole 64-bit words."""
    bits = d if k_bits == 0 else k_bits
    if bits <= 0 or d % bits:
        raise ValueError(f"Sign-OPORP bins the {d} coordinates into k_bits equal groups: {bits} does not divide {d}")
    if bits % 64:
        raise ValueError(f"Sign-OPORP codes are packed in 64-bit words: k_bits={bits} is not a multiple of 64")
    return bits


def _oporp_draws(d: int, seed: int, device: torch.device) -> tuple[Tensor, Tensor]:
    """The random sign flips (int8 +-1) and the coordinate permutation, drawn in that order
    from one generator seeded with ``seed`` on ``device`` (the reference's order,
    indexing/quantize.py:55-60: a ``randint`` then a ``randperm``)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    flips = torch.randint(0, 2, (d,), generator=gen, device=device, dtype=torch.int8) * 2 - 1
    order = torch.randperm(d, generator=gen, device=device)
    return flips, order


def _oporp_sketch(rows: Tensor, flips: Tensor, order: Tensor, n_bits: int) -> Tensor:
    """Flip, permute, sum each run of ``D / n_bits`` consecutive coordinates into one bin, and
    scale every row to unit norm (norms below 1e-8 taken as 1e-8): the reference's arithmetic
    (indexing/quantize.py:97-105), so each bin's sign is the reference's bit."""
    permuted = (rows * flips.to(rows.dtype))[:, order]
    bins = permuted.reshape(rows.shape[0], n_bits, -1).sum(dim=-1)
    return bins / bins.norm(dim=-1, keepdim=True).clamp_min(1e-8)


def quantize_oporp_1bit(embs: Tensor, seed: int = 0, k_bits: int = 0) -> tuple[Tensor, Tensor, Tensor]:
    """Sign-OPORP codes ``(bits [N, k_bits // 64] int64, signs [D] int8, perm [D] int64)``."""
    _matrix(embs, "embs")
    n_bits = _oporp_bits(embs.shape[1], k_bits)
    flips, order = _oporp_draws(embs.shape[1], seed, embs.device)
    return _codes(embs, n_bits, lambda rows: _oporp_sketch(rows, flips, order, n_bits)), flips, order


def project_oporp_1bit_query(query: Tensor, signs: Tensor, perm: Tensor, k_bits: int = 0) -> Tensor:
    """A query batch's Sign-OPORP code under the table's ``signs`` and ``perm``."""
    _matrix(query, "query")
    return pack_signs(_oporp_sketch(query, signs, perm, _oporp_bits(query.shape[1], k_bits)))
