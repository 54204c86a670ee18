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

_CHUNK_ROWS = 1 << 16  # rows projected at a time in the 1-bit builds


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


def _pack_chunked(embs: Tensor, w: int, project) -> Tensor:
    bits = torch.empty((embs.shape[0], w), dtype=torch.int64, device=embs.device)
    for start in range(0, embs.shape[0], _CHUNK_ROWS):
        bits[start : start + _CHUNK_ROWS] = pack_signs(project(embs[start : start + _CHUNK_ROWS]))
    return bits


def _simhash_r(d: int, k_bits: int, seed: int, device: torch.device) -> Tensor:
    g = torch.Generator(device=device).manual_seed(int(seed))
    return torch.randn(k_bits, d, generator=g, device=device)


def quantize_simhash_1bit(embs: Tensor, k_bits: int, seed: int = 0) -> tuple[Tensor, Tensor]:
    """SimHash codes ``(bits [N, k_bits // 64] int64, r [k_bits, D] fp32)``."""
    if embs.dim() != 2:
        raise ValueError(f"expected 2-D [N, D] embeddings, got shape {tuple(embs.shape)}")
    if k_bits % 64 != 0:
        raise ValueError(f"k_bits must be a multiple of 64, got {k_bits}")
    _cuda(embs)
    r = _simhash_r(embs.shape[1], k_bits, seed, embs.device)
    return _pack_chunked(embs, k_bits // 64, lambda x: x @ r.t()), r


def project_simhash_1bit_query(query: Tensor, r: Tensor) -> Tensor:
    """The same projection for a query batch: ``[B, k_bits // 64]`` int64."""
    if query.dim() != 2:
        raise ValueError(f"expected 2-D [B, D] query, got shape {tuple(query.shape)}")
    _cuda(query)
    return pack_signs(query @ r.t())


def _oporp_k_bits(d: int, k_bits: int) -> int:
    if k_bits == 0:
        k_bits = d
    if d % k_bits != 0:
        raise ValueError(f"k_bits must divide D; got k_bits={k_bits}, D={d}")
    if k_bits % 64 != 0:
        raise ValueError(f"k_bits (D when 0) must be a multiple of 64, got {k_bits}")
    return k_bits


def _oporp_params(d: int, seed: int, device: torch.device) -> tuple[Tensor, Tensor]:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    signs = torch.randint(0, 2, (d,), generator=g, device=device, dtype=torch.int8) * 2 - 1
    perm = torch.randperm(d, generator=g, device=device)
    return signs, perm


def _oporp_sketch(x: Tensor, signs: Tensor, perm: Tensor, k_bits: int) -> Tensor:
    n, d = x.shape
    proj = (x * signs.to(x.dtype)).index_select(1, perm)
    binned = proj.view(n, k_bits, d // k_bits).sum(dim=-1)
    return binned / binned.norm(dim=-1, keepdim=True).clamp_min(1e-8)


def quantize_oporp_1bit(embs: Tensor, seed: int = 0, k_bits: int = 0) -> tuple[Tensor, Tensor, Tensor]:
    """Sign-OPORP codes ``(bits [N, k_bits // 64] int64, signs [D] int8, perm [D] int64)``."""
    if embs.dim() != 2:
        raise ValueError(f"expected 2-D [N, D] embeddings, got shape {tuple(embs.shape)}")
    _cuda(embs)
    k_bits = _oporp_k_bits(embs.shape[1], k_bits)
    signs, perm = _oporp_params(embs.shape[1], seed, embs.device)
    bits = _pack_chunked(embs, k_bits // 64, lambda x: _oporp_sketch(x, signs, perm, k_bits))
    return bits, signs, perm


def project_oporp_1bit_query(query: Tensor, signs: Tensor, perm: Tensor, k_bits: int = 0) -> Tensor:
    """The same Sign-OPORP projection for a query batch."""
    if query.dim() != 2:
        raise ValueError(f"expected 2-D [B, D] query, got shape {tuple(query.shape)}")
    _cuda(query)
    return pack_signs(_oporp_sketch(query, signs, perm, _oporp_k_bits(query.shape[1], k_bits)))
