"""The ``retrieve::*`` op namespace backed by ``libretrieve_b200.so``.

This module is the drop-in for ``retrieve.ops.triton`` (the package
``retrieve.interfaces.ops_for("triton")`` imports,
retrieve/src/retrieve/interfaces.py:25-37): the same op names and signatures,
registered as ``torch.ops.retrieve.<name>`` with fake (meta) implementations,
plus ``dense_topk``, the fused score + top-k the reference runs as
``torch.mm`` + ``torch.topk`` (retrieve/src/retrieve/modules/knn.py:62-76).

Every op runs on the caller's current CUDA stream, allocates its outputs and
scratch through the torch caching allocator, never synchronises the host and
raises ``ValueError`` / ``TypeError`` for bad inputs like the reference
(retrieve/src/retrieve/ops/triton/_host.py:25-31). There is no CPU path: CPU
tensors raise.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from retrieve_b200 import _lib

_DTYPE_CODE = {torch.float16: _lib.RB_F16, torch.bfloat16: _lib.RB_BF16}


def _stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _require_cuda(*tensors: Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("retrieve_b200 ops run on CUDA tensors only")


def check_contiguous(**tables: Tensor) -> None:
    """Item-side tables must arrive contiguous (a per-call copy would copy the
    whole index every forward; retrieve/src/retrieve/ops/triton/_host.py:25-31)."""
    for name, t in tables.items():
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous (copy it once at index build)")


# ---------------------------------------------------------------------------
# dense_topk
# ---------------------------------------------------------------------------
def _dense_topk_impl(query: Tensor, item_embs: Tensor, k: int, id_offset: int = 0) -> tuple[Tensor, Tensor]:
    if query.dim() != 2 or item_embs.dim() != 2:
        raise ValueError("query must be [B, D] and item_embs [N, D]")
    if item_embs.dtype not in _DTYPE_CODE:
        raise TypeError(f"item_embs must be float16 or bfloat16, got {item_embs.dtype}")
    if query.shape[1] != item_embs.shape[1]:
        raise ValueError(f"D mismatch: query D={query.shape[1]} vs item_embs D={item_embs.shape[1]}")
    if k < 1:
        raise ValueError(f"k must be positive, got {k}")
    _require_cuda(query, item_embs)
    check_contiguous(item_embs=item_embs)
    q = query.to(item_embs.dtype).contiguous()
    b, d = q.shape
    n = item_embs.shape[0]
    dev = q.device
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    lib = _lib.lib()
    code = _DTYPE_CODE[item_embs.dtype]
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_workspace_size(b, n, d, code, k, ctypes.byref(nbytes)), "dense_topk")
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.rb_dense_topk(
            _ptr(q), _ptr(item_embs), b, n, d, code, k, int(id_offset), _ptr(ids), _ptr(scores),
            _ptr(ws), ws.numel(), _stream_ptr(dev),
        )
    _lib.check(rc, "dense_topk")
    return ids, scores


@torch.library.custom_op("retrieve::dense_topk", mutates_args=(), device_types="cuda")
def dense_topk(query: Tensor, item_embs: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """Fused ``query @ item_embs.T`` (fp32 accumulation on the tensor cores) +
    top-``k`` → ``(ids [B, k] int64, scores [B, k] fp32)``, sorted by score
    descending, ties to the lower id, ``-1`` / ``-inf`` past the corpus size.
    ``item_embs`` is ``[N, D]`` fp16 or bf16 and contiguous; the query is cast to
    its dtype (the reference casts to fp16, knn.py:64). The ``[B, N]`` score
    matrix of the reference path is never materialised."""
    return _dense_topk_impl(query, item_embs, k)


@dense_topk.register_fake
def _(query, item_embs, k):
    b = query.shape[0]
    return (
        query.new_empty((b, k), dtype=torch.int64),
        query.new_empty((b, k), dtype=torch.float32),
    )


def dense_topk_sharded(query: Tensor, item_shard: Tensor, k: int, id_offset: int) -> tuple[Tensor, Tensor]:
    """``dense_topk`` over one row shard of a larger corpus: ids come back global
    (``id_offset`` + local row). Used by :mod:`retrieve_b200.shard`."""
    return _dense_topk_impl(query, item_shard, k, id_offset)


__all__ = ["check_contiguous", "dense_topk", "dense_topk_sharded"]
