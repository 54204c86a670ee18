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
def _dense_topk_impl(
    query: Tensor, item_embs: Tensor, k: int, id_offset: int = 0, ws: Tensor | None = None
) -> tuple[Tensor, Tensor]:
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
    if ws is None or ws.numel() < nbytes.value:
        ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.rb_dense_topk(
            _ptr(q), _ptr(item_embs), b, n, d, code, k, int(id_offset), _ptr(ids), _ptr(scores),
            _ptr(ws), ws.numel(), _stream_ptr(dev),
        )
    _lib.check(rc, "dense_topk")
    return ids, scores


def dense_workspace(query: Tensor, item_shard: Tensor, k: int) -> Tensor:
    """Device workspace for the dense top-k entry points on this shard."""
    b, d = query.shape
    nbytes = ctypes.c_size_t(0)
    _lib.check(
        _lib.lib().rb_dense_topk_workspace_size(b, item_shard.shape[0], d, _DTYPE_CODE[item_shard.dtype], k,
                                                ctypes.byref(nbytes)),
        "dense_topk",
    )
    return torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=query.device)


def dense_seed_sample(
    query: Tensor, item_shard: Tensor, k: int, n_total: int, ws: Tensor | None = None, m: int | None = None
) -> Tensor:
    """Per query, this shard's top ``m`` (default k) sampled tile maxima
    (``[B, m]`` fp32) for the threshold shared by all shards (C-ABI
    ``rb_dense_seed_sample``)."""
    m = k if m is None else int(m)
    _require_cuda(query, item_shard)
    check_contiguous(item_shard=item_shard)
    q = query.to(item_shard.dtype).contiguous()
    b, d = q.shape
    dev = q.device
    out = torch.empty((b, m), dtype=torch.float32, device=dev)
    if b == 0:
        return out
    ws = dense_workspace(q, item_shard, k) if ws is None else ws
    with torch.cuda.device(dev):
        rc = _lib.lib().rb_dense_seed_sample(
            _ptr(q), _ptr(item_shard), b, item_shard.shape[0], d, _DTYPE_CODE[item_shard.dtype], k, m, int(n_total),
            _ptr(out), _ptr(ws), ws.numel(), _stream_ptr(dev),
        )
    _lib.check(rc, "dense_seed_sample")
    return out


def dense_topk_seeded(
    query: Tensor, item_shard: Tensor, k: int, id_offset: int, n_total: int, seed_vals: Tensor,
    ws: Tensor | None = None, pairs: bool = False,
) -> tuple[Tensor, Tensor] | Tensor:
    """``dense_topk_sharded`` with the full pass seeded by the union of every
    shard's ``dense_seed_sample`` output (``seed_vals [W, B, m]`` fp32; C-ABI
    ``rb_dense_topk_seeded``). May return fewer than k real entries per row
    (``-1`` / ``-inf``); the merge over all shards is the exact global top-k.
    With ``pairs`` the result is one ``[B, k]`` int64 tensor of packed (fp32
    score bits, uint32 global id) pairs for ``merge_pairs``."""
    _require_cuda(query, item_shard)
    check_contiguous(item_shard=item_shard, seed_vals=seed_vals)
    q = query.to(item_shard.dtype).contiguous()
    b, d = q.shape
    if seed_vals.dim() != 3 or seed_vals.shape[1] != b or not 1 <= seed_vals.shape[2] <= k \
            or seed_vals.dtype != torch.float32:
        raise ValueError("seed_vals must be [W, B, m] float32 with 1 <= m <= k")
    dev = q.device
    if pairs:
        out = torch.empty((b, k), dtype=torch.int64, device=dev)
        ids = scores = None
    else:
        out = None
        ids = torch.empty((b, k), dtype=torch.int64, device=dev)
        scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b > 0:
        ws = dense_workspace(q, item_shard, k) if ws is None else ws
        with torch.cuda.device(dev):
            rc = _lib.lib().rb_dense_topk_seeded(
                _ptr(q), _ptr(item_shard), b, item_shard.shape[0], d, _DTYPE_CODE[item_shard.dtype], k,
                int(id_offset), int(n_total), _ptr(seed_vals), seed_vals.shape[0], seed_vals.shape[2],
                None if pairs else _ptr(ids), None if pairs else _ptr(scores), _ptr(out) if pairs else None,
                _ptr(ws), ws.numel(), _stream_ptr(dev),
            )
        _lib.check(rc, "dense_topk_seeded")
    return out if pairs else (ids, scores)


def merge_pairs(pairs: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """``[W, B, kin]`` packed (score bits, uint32 id) pairs of every shard →
    global ``(ids [B, k] int64, scores [B, k] fp32)`` (C-ABI ``rb_merge_pairs``)."""
    if pairs.dim() != 3 or pairs.dtype != torch.int64:
        raise ValueError("pairs must be [W, B, kin] int64")
    _require_cuda(pairs)
    check_contiguous(pairs=pairs)
    w, b, kin = pairs.shape
    dev = pairs.device
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    with torch.cuda.device(dev):
        rc = _lib.lib().rb_merge_pairs(_ptr(pairs), w, b, kin, k, _ptr(ids), _ptr(scores), _stream_ptr(dev))
    _lib.check(rc, "merge_pairs")
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


def dense_topk_sharded(
    query: Tensor, item_shard: Tensor, k: int, id_offset: int, ws: Tensor | None = None
) -> tuple[Tensor, Tensor]:
    """``dense_topk`` over one row shard of a larger corpus: ids come back global
    (``id_offset`` + local row); ``ws``, if large enough, is the device workspace
    (``dense_workspace``). Used by :mod:`retrieve_b200.shard`."""
    return _dense_topk_impl(query, item_shard, k, id_offset, ws)


# ---------------------------------------------------------------------------
# dense_topk with an attribute predicate (LiNR V1 with its filter; bloom scan)
# ---------------------------------------------------------------------------
FILTER_MODES = {"exact": 1, "bloom": 2, "bloom_recheck": 3}


class _RbFilter(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int),
        ("terms", ctypes.c_void_p),
        ("n_terms", ctypes.c_void_p),
        ("item_attrs", ctypes.c_void_p),
        ("n_clauses", ctypes.c_int),
        ("attr_width", ctypes.c_int),
        ("item_bloom", ctypes.c_void_p),
        ("item_bloom_slices", ctypes.c_void_p),
    ]


@torch.library.custom_op("retrieve::dense_topk_filtered", mutates_args=(), device_types="cuda")
def dense_topk_filtered(
    query: Tensor,
    item_embs: Tensor,
    k: int,
    terms: Tensor,
    n_terms: Tensor,
    mode: str,
    item_attrs: Tensor | None = None,
    item_bloom: Tensor | None = None,
    item_bloom_slices: Tensor | None = None,
) -> tuple[Tensor, Tensor]:
    """``dense_topk`` over the items that pass each query's predicate
    (``retrieve_b200.predicates``): ``mode`` ``"exact"`` tests ``item_attrs
    [N, C, A]`` int64, ``"bloom"`` the per-item 64-bit words ``item_bloom [N]``
    (false positives possible, no false negatives for NOT-free predicates),
    ``"bloom_recheck"`` both. Rows with fewer than k passing items end in
    ``-1`` / ``-inf``. The predicate is evaluated inside the fused scan, only on
    items whose score already clears the running top-k threshold.
    ``item_bloom_slices`` (optional, the Bloom modes): ``bloom_slices(item_bloom)``
    built once with the index; without it the call builds them into its workspace."""
    if mode not in FILTER_MODES:
        raise ValueError(f"mode must be one of {sorted(FILTER_MODES)}, got {mode!r}")
    if query.dim() != 2 or item_embs.dim() != 2:
        raise ValueError("query must be [B, D] and item_embs [N, D]")
    if item_embs.dtype not in _DTYPE_CODE:
        raise TypeError(f"item_embs must be float16 or bfloat16, got {item_embs.dtype}")
    b, n = query.shape[0], item_embs.shape[0]
    if terms.shape != (b, 8 * 24) or terms.dtype != torch.uint8 or n_terms.shape != (b,):
        raise ValueError("terms must be [B, 192] uint8 and n_terms [B] int32 (retrieve_b200.predicates)")
    _require_cuda(query, item_embs, terms, n_terms)
    check_contiguous(item_embs=item_embs)
    m = FILTER_MODES[mode]
    attrs = None
    if m in (1, 3):
        if item_attrs is None or item_attrs.dim() != 3 or item_attrs.dtype != torch.int64:
            raise ValueError("exact filtering needs item_attrs [N, C, A] int64")
        if item_attrs.shape[0] != n:
            raise ValueError("item_attrs must have one row per item")
        check_contiguous(item_attrs=item_attrs)
        attrs = item_attrs
    if m in (2, 3):
        if item_bloom is None or item_bloom.shape != (n,) or item_bloom.dtype not in (torch.int64, torch.uint64):
            raise ValueError("bloom filtering needs item_bloom [N] 64-bit words")
        check_contiguous(item_bloom=item_bloom)
        if item_bloom_slices is not None:
            if (item_bloom_slices.dim() != 1 or item_bloom_slices.dtype != torch.int32
                    or item_bloom_slices.numel() < (n + 127) // 128 * 256):
                raise ValueError("item_bloom_slices must be bloom_slices(item_bloom): int32, 256 words per 128 items")
            _require_cuda(item_bloom_slices)
            check_contiguous(item_bloom_slices=item_bloom_slices)
    q = query.to(item_embs.dtype).contiguous()
    tt = terms.contiguous()
    nt = n_terms.to(torch.int32).contiguous()
    dev = q.device
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    f = _RbFilter(
        m, tt.data_ptr(), nt.data_ptr(), 0 if attrs is None else attrs.data_ptr(),
        0 if attrs is None else attrs.shape[1], 0 if attrs is None else attrs.shape[2],
        0 if item_bloom is None else item_bloom.data_ptr(),
        0 if item_bloom_slices is None or m not in (2, 3) else item_bloom_slices.data_ptr(),
    )
    lib = _lib.lib()
    code = _DTYPE_CODE[item_embs.dtype]
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_filtered_workspace_size(b, n, q.shape[1], code, k, m, ctypes.byref(nb)),
               "dense_topk_filtered")
    ws = torch.empty(max(int(nb.value), 256), dtype=torch.uint8, device=dev)
    rc = lib.rb_dense_topk_filtered(_ptr(q), _ptr(item_embs), b, n, q.shape[1], code, k, 0, ctypes.addressof(f),
                                    _ptr(ids), _ptr(scores), _ptr(ws), ws.numel(), _stream_ptr(dev))
    _lib.check(rc, "dense_topk_filtered")
    return ids, scores


@dense_topk_filtered.register_fake
def _(query, item_embs, k, terms, n_terms, mode, item_attrs=None, item_bloom=None, item_bloom_slices=None):
    b = query.shape[0]
    return query.new_empty((b, k), dtype=torch.int64), query.new_empty((b, k), dtype=torch.float32)


def bloom_build(item_attrs: Tensor, k: int = 3) -> Tensor:
    """Per-item 64-bit Bloom words (int64 view of the uint64 words) of
    ``item_attrs [N, C, A]`` int64 (``rb_bloom_build``). Build time."""
    if item_attrs.dim() != 3 or item_attrs.dtype != torch.int64:
        raise ValueError("item_attrs must be [N, C, A] int64")
    _require_cuda(item_attrs)
    a = item_attrs.contiguous()
    out = torch.empty((a.shape[0],), dtype=torch.int64, device=a.device)
    rc = _lib.lib().rb_bloom_build(_ptr(a), a.shape[0], a.shape[1], a.shape[2], k, _ptr(out), _stream_ptr(a.device))
    _lib.check(rc, "bloom_build")
    return out


def bloom_slices(item_bloom: Tensor) -> Tensor:
    """The per-item Bloom words ``item_bloom [N]`` (``bloom_build``) bit-sliced for the
    filtered scans (``rb_bloom_slices``): per 32-item chunk 64 int32 words, word p
    holding bit p of the chunk's items, whole 128-item tiles. Build time; pass the
    result to ``dense_topk_filtered(..., item_bloom_slices=...)``."""
    if item_bloom.dim() != 1 or item_bloom.dtype != torch.int64:
        raise ValueError("item_bloom must be [N] int64 (bloom_build)")
    _require_cuda(item_bloom)
    w = item_bloom.contiguous()
    nb = ctypes.c_size_t(0)
    lib = _lib.lib()
    _lib.check(lib.rb_bloom_slices_bytes(w.shape[0], ctypes.byref(nb)), "bloom_slices")
    out = torch.zeros((max(int(nb.value) // 4, 4),), dtype=torch.int32, device=w.device)
    _lib.check(lib.rb_bloom_slices(_ptr(w), w.shape[0], _ptr(out), _stream_ptr(w.device)), "bloom_slices")
    return out


# ---------------------------------------------------------------------------
# clause filter (retrieve/src/retrieve/ops/triton/clause_mask.py,
# clause_compact.py; predicate functional.py:173-185)
# ---------------------------------------------------------------------------
def _clause_prep(item_clause_attrs: Tensor, clause_is_reverse: Tensor, query_clause_attrs: Tensor):
    """Validation + contiguity, as ``_clause_mask_prep`` (clause_mask.py:150-183)."""
    if item_clause_attrs.dim() != 3:
        raise ValueError("item_clause_attrs must be [N, C, A_max]")
    if query_clause_attrs.dim() != 2:
        raise ValueError("query_clause_attrs must be [B, C]")
    n, c, a_max = item_clause_attrs.shape
    b, c_q = query_clause_attrs.shape
    if c != c_q:
        raise ValueError(f"clause-count mismatch: items C={c}, query C={c_q}")
    if item_clause_attrs.dtype != torch.int64:
        raise TypeError(f"item_clause_attrs must be int64, got {item_clause_attrs.dtype}")
    if b > 65535:
        raise ValueError("the clause kernels take at most 65535 query rows per call")
    _require_cuda(item_clause_attrs, query_clause_attrs)
    check_contiguous(item_clause_attrs=item_clause_attrs)
    rev = clause_is_reverse.to(device=item_clause_attrs.device, dtype=torch.uint8).contiguous()
    if rev.numel() != c:
        raise ValueError(f"clause_is_reverse must have {c} entries, got {rev.numel()}")
    qa = query_clause_attrs.to(torch.int64).contiguous()
    return item_clause_attrs, rev, qa, b, n, c, a_max


@torch.library.custom_op("retrieve::clause_mask", mutates_args=(), device_types="cuda")
def clause_mask(item_clause_attrs: Tensor, clause_is_reverse: Tensor, query_clause_attrs: Tensor) -> Tensor:
    """Exact clause evaluation → ``[B, N]`` bool (clause_mask.py:270-283)."""
    attrs, rev, qa, b, n, c, a = _clause_prep(item_clause_attrs, clause_is_reverse, query_clause_attrs)
    out = torch.empty((b, n), dtype=torch.bool, device=attrs.device)
    if b and n:
        rc = _lib.lib().rb_clause_mask(_ptr(attrs), n, c, a, _ptr(rev), _ptr(qa), b, None, _ptr(out),
                                       _stream_ptr(attrs.device))
        _lib.check(rc, "clause_mask")
    return out


@clause_mask.register_fake
def _(item_clause_attrs, clause_is_reverse, query_clause_attrs):
    return query_clause_attrs.new_empty((query_clause_attrs.shape[0], item_clause_attrs.shape[0]), dtype=torch.bool)


@torch.library.custom_op("retrieve::clause_mask_scores", mutates_args=(), device_types="cuda")
def clause_mask_scores(
    scores: Tensor, item_clause_attrs: Tensor, clause_is_reverse: Tensor, query_clause_attrs: Tensor
) -> Tensor:
    """``where(clause_mask(...), scores, -inf)`` in one pass (clause_mask.py:286-303)."""
    attrs, rev, qa, b, n, c, a = _clause_prep(item_clause_attrs, clause_is_reverse, query_clause_attrs)
    if scores.shape != (b, n) or scores.dtype != torch.float32:
        raise ValueError(f"scores must be [B, N] = {[b, n]} float32, got {scores.shape} {scores.dtype}")
    sc = scores.contiguous()
    out = torch.empty((b, n), dtype=torch.float32, device=attrs.device)
    if b and n:
        rc = _lib.lib().rb_clause_mask(_ptr(attrs), n, c, a, _ptr(rev), _ptr(qa), b, _ptr(sc), _ptr(out),
                                       _stream_ptr(attrs.device))
        _lib.check(rc, "clause_mask_scores")
    return out


@clause_mask_scores.register_fake
def _(scores, item_clause_attrs, clause_is_reverse, query_clause_attrs):
    return torch.empty_like(scores)


@torch.library.custom_op("retrieve::clause_compact", mutates_args=(), device_types="cuda")
def clause_compact(
    item_clause_attrs: Tensor, clause_is_reverse: Tensor, query_clause_attrs: Tensor
) -> tuple[Tensor, Tensor]:
    """Clause evaluation + compaction → ``(positive_indices [B, N] int64, counts
    [B] int64)``: each row's passing ids in ascending order on ``[0, counts[b])``,
    the tail unwritten (clause_compact.py:174-196)."""
    attrs, rev, qa, b, n, c, a = _clause_prep(item_clause_attrs, clause_is_reverse, query_clause_attrs)
    ids = torch.empty((b, n), dtype=torch.int64, device=attrs.device)
    counts = torch.empty((b,), dtype=torch.int64, device=attrs.device)
    if b:
        lib = _lib.lib()
        nb = ctypes.c_size_t(0)
        _lib.check(lib.rb_clause_compact_workspace_size(b, n, ctypes.byref(nb)), "clause_compact")
        ws = torch.empty(max(int(nb.value), 256), dtype=torch.uint8, device=attrs.device)
        rc = lib.rb_clause_compact(_ptr(attrs), n, c, a, _ptr(rev), _ptr(qa), b, _ptr(ids), _ptr(counts), _ptr(ws),
                                   ws.numel(), _stream_ptr(attrs.device))
        _lib.check(rc, "clause_compact")
    return ids, counts


@clause_compact.register_fake
def _(item_clause_attrs, clause_is_reverse, query_clause_attrs):
    b, n = query_clause_attrs.shape[0], item_clause_attrs.shape[0]
    return (
        query_clause_attrs.new_empty((b, n), dtype=torch.int64),
        query_clause_attrs.new_empty((b,), dtype=torch.int64),
    )


# ---------------------------------------------------------------------------
# gemv_scores (ops/triton/gemv_scores.py:31-43)
# ---------------------------------------------------------------------------
@torch.library.custom_op("retrieve::gemv_scores", mutates_args=(), device_types="cuda")
def gemv_scores(query: Tensor, item_embs_t: Tensor) -> Tensor:
    """``query [1, D]`` fp16 against ``item_embs_t [D, N]`` fp16 (contiguous) →
    ``[1, N]`` fp32, one fp32 FMA per k in order (the order of cuBLAS's gemv2N)."""
    if query.shape[0] != 1 or query.dtype != torch.float16 or item_embs_t.dtype != torch.float16:
        raise ValueError("gemv_scores takes one fp16 query row and an fp16 [D, N] table")
    _require_cuda(query, item_embs_t)
    check_contiguous(item_embs_t=item_embs_t)
    d, n = item_embs_t.shape
    q = query.contiguous()
    out = torch.empty((1, n), dtype=torch.float32, device=q.device)
    rc = _lib.lib().rb_gemv_scores(_ptr(q), _ptr(item_embs_t), d, n, _ptr(out), _stream_ptr(q.device))
    _lib.check(rc, "gemv_scores")
    return out


@gemv_scores.register_fake
def _(query, item_embs_t):
    return query.new_empty((1, item_embs_t.shape[1]), dtype=torch.float32)


# ---------------------------------------------------------------------------
# candidate top-k: fused_masked_knn_topk / oporp indirect
# ---------------------------------------------------------------------------
_CAND_DTYPES = {torch.float16: _lib.RB_F16, torch.float32: _lib.RB_F32}


def _candidate_topk(kind, query, items, positive_indices, counts, k, k_out):
    lib = _lib.lib()
    b, p = positive_indices.shape
    dev = query.device
    ids = torch.empty((b, k_out), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k_out), dtype=torch.float32, device=dev)
    if b == 0 or k_out == 0:
        return ids, scores
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_candidate_topk_workspace_size(b, p, ctypes.byref(nb)), "candidate_topk")
    ws = torch.empty(max(int(nb.value), 256), dtype=torch.uint8, device=dev)
    qd = _CAND_DTYPES.get(query.dtype, _lib.RB_F32)
    xd = _CAND_DTYPES.get(items.dtype, _lib.RB_F32)
    rc = lib.rb_candidate_topk(
        kind, _ptr(query), qd, _ptr(items), xd, items.shape[0], query.shape[1], _ptr(positive_indices), p,
        _ptr(counts), b, k, _ptr(ids), _ptr(scores), _ptr(ws), ws.numel(), _stream_ptr(dev),
    )
    _lib.check(rc, "candidate_topk")
    return ids, scores


@torch.library.custom_op("retrieve::fused_masked_knn_topk", mutates_args=(), device_types="cuda")
def fused_masked_knn_topk(
    query: Tensor, item_embs: Tensor, positive_indices: Tensor, counts: Tensor, k: int
) -> tuple[Tensor, Tensor]:
    """Fused gather + fp32 dot + top-k over ``positive_indices[b, :counts[b]]`` →
    ``(ids [B, k], scores [B, k])``; requires ``P >= k`` (``ValueError``
    otherwise, as the reference op, fused_masked_knn_topk.py:289-310); rows
    short of candidates end in ``-1`` / ``-inf``."""
    if positive_indices.shape[1] < k:
        raise ValueError(f"positive_indices has {positive_indices.shape[1]} columns, fewer than k={k}")
    if query.dim() != 2 or item_embs.dim() != 2:
        raise ValueError("query must be [B, D] and item_embs [N, D]")
    if query.dtype not in _CAND_DTYPES or item_embs.dtype not in _CAND_DTYPES:
        raise TypeError(
            f"query and item_embs must be float16 or float32, got {query.dtype} and {item_embs.dtype}"
        )
    if query.shape[1] != item_embs.shape[1]:
        raise ValueError("query and item_embs must have the same D")
    _require_cuda(query, item_embs, positive_indices, counts)
    check_contiguous(item_embs=item_embs, positive_indices=positive_indices)
    return _candidate_topk(
        0, query.contiguous(), item_embs, positive_indices.to(torch.int64), counts.to(torch.int64).contiguous(),
        k, k,
    )


@fused_masked_knn_topk.register_fake
def _(query, item_embs, positive_indices, counts, k):
    b = query.shape[0]
    return query.new_empty((b, k), dtype=torch.int64), query.new_empty((b, k), dtype=torch.float32)


def _oporp_check(query_bits: Tensor, item_bits: Tensor) -> None:
    """As ``_oporp_prep`` (oporp_1bit_match_topk.py:134-163)."""
    if query_bits.dim() != 2 or item_bits.dim() != 2:
        raise ValueError("query_bits must be [B, W] and item_bits [N, W]")
    if query_bits.dtype != torch.int64 or item_bits.dtype != torch.int64:
        raise TypeError("query_bits and item_bits must be int64")
    if query_bits.shape[1] != item_bits.shape[1]:
        raise ValueError(
            f"W mismatch: query_bits W={query_bits.shape[1]} vs item_bits W={item_bits.shape[1]}"
        )
    _require_cuda(query_bits, item_bits)
    check_contiguous(item_bits=item_bits)


@torch.library.custom_op("retrieve::oporp_1bit_match_topk_full", mutates_args=(), device_types="cuda")
def oporp_1bit_match_topk_full(query_bits: Tensor, item_bits: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """Full-scan 1-bit Hamming top-k: score ``64*W - 2*popcount(q ^ item)`` over
    every row of ``item_bits`` → ``(ids [B, k], scores [B, k])``, ties to the
    lower row (oporp_1bit_match_topk.py:261-273)."""
    _oporp_check(query_bits, item_bits)
    b, w = query_bits.shape
    n = item_bits.shape[0]
    if k > n:
        raise RuntimeError(f"selected index k={k} out of range for {n} items")
    q = query_bits.contiguous()
    dev = q.device
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    lib = _lib.lib()
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_hamming_topk_workspace_size(b, n, w, k, ctypes.byref(nb)), "oporp_1bit_match_topk_full")
    ws = torch.empty(max(int(nb.value), 256), dtype=torch.uint8, device=dev)
    rc = lib.rb_hamming_topk(_ptr(q), _ptr(item_bits), b, n, w, k, _ptr(ids), _ptr(scores), _ptr(ws), ws.numel(),
                             _stream_ptr(dev))
    _lib.check(rc, "oporp_1bit_match_topk_full")
    return ids, scores


@oporp_1bit_match_topk_full.register_fake
def _(query_bits, item_bits, k):
    b = query_bits.shape[0]
    return query_bits.new_empty((b, k), dtype=torch.int64), query_bits.new_empty((b, k), dtype=torch.float32)


@torch.library.custom_op("retrieve::oporp_1bit_match_topk_indirect", mutates_args=(), device_types="cuda")
def oporp_1bit_match_topk_indirect(
    query_bits: Tensor, item_bits: Tensor, k: int, positive_indices: Tensor, counts: Tensor
) -> tuple[Tensor, Tensor]:
    """Hamming top-k over ``positive_indices[b, :counts[b]]`` only; returns
    ``min(k, P)`` columns with ``-1`` / ``-inf`` where a row runs out of
    candidates (oporp_1bit_match_topk.py:276-292)."""
    _oporp_check(query_bits, item_bits)
    _require_cuda(positive_indices, counts)
    check_contiguous(positive_indices=positive_indices)
    p = positive_indices.shape[1]
    return _candidate_topk(
        1, query_bits.contiguous(), item_bits, positive_indices.to(torch.int64),
        counts.to(torch.int64).contiguous(), k, min(k, p),
    )


@oporp_1bit_match_topk_indirect.register_fake
def _(query_bits, item_bits, k, positive_indices, counts):
    b, p = positive_indices.shape
    kk = min(k, p)
    return query_bits.new_empty((b, kk), dtype=torch.int64), query_bits.new_empty((b, kk), dtype=torch.float32)


# ---------------------------------------------------------------------------
# query-side int8 quantization (indexing/quantize.py:9-18)
# ---------------------------------------------------------------------------
@torch.library.custom_op("retrieve::quantize_int8", mutates_args=(), device_types="cuda")
def quantize_int8(embs: Tensor) -> tuple[Tensor, Tensor]:
    """Per-row symmetric int8 codes and fp32 scales, bit for bit
    ``retrieve.indexing.quantize.quantize_int8``."""
    if embs.dim() != 2:
        raise ValueError(f"expected 2-D [B, D] input, got shape {tuple(embs.shape)}")
    _require_cuda(embs)
    x = embs.to(torch.float32).contiguous()
    b, d = x.shape
    codes = torch.empty((b, d), dtype=torch.int8, device=x.device)
    scales = torch.empty((b,), dtype=torch.float32, device=x.device)
    if b:
        rc = _lib.lib().rb_quantize_int8(_ptr(x), b, d, _ptr(codes), _ptr(scales), _stream_ptr(x.device))
        _lib.check(rc, "quantize_int8")
    return codes, scales


@quantize_int8.register_fake
def _(embs):
    return embs.new_empty(embs.shape, dtype=torch.int8), embs.new_empty((embs.shape[0],), dtype=torch.float32)


# ---------------------------------------------------------------------------
# int8 scoring (SilverTorch's int32 scoring path)
# ---------------------------------------------------------------------------
@torch.library.custom_op("retrieve::int8_topk", mutates_args=(), device_types="cuda")
def int8_topk(query: Tensor, item_codes: Tensor, item_scales: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """Int8 scoring + top-k: the fp32 query batch is quantized per row exactly as
    ``quantize_int8`` (indexing/quantize.py:9-18), scored against ``item_codes
    [N, D]`` int8 with int32 accumulation on the tensor cores, and dequantized as
    ``(fp32(dot) * q_scale) * item_scale`` (the reference's order,
    ops/official/adapter.py:338-367). ``item_scales`` is ``[N]`` fp32 (all equal
    for SilverTorch's global scale). Ties go to the lower item id."""
    if query.dim() != 2 or item_codes.dim() != 2:
        raise ValueError("query must be [B, D] and item_codes [N, D]")
    if item_codes.dtype != torch.int8:
        raise TypeError(f"item_codes must be int8, got {item_codes.dtype}")
    if item_scales.dim() != 1 or item_scales.shape[0] != item_codes.shape[0]:
        raise ValueError("item_scales must be [N]")
    if query.shape[1] != item_codes.shape[1]:
        raise ValueError("query and item_codes must have the same D")
    _require_cuda(query, item_codes, item_scales)
    check_contiguous(item_codes=item_codes, item_scales=item_scales)
    xs = item_scales.to(torch.float32).contiguous()
    codes, qs = quantize_int8(query)
    return int8_codes_topk(codes, qs, item_codes, xs, k)


def scaled_topk(
    queries: Tensor, query_scales: Tensor | None, items: Tensor, item_scales: Tensor | None, k: int, dtype_code: int,
    id_offset: int = 0,
) -> tuple[Tensor, Tensor]:
    """Dense top-k over fp8 e4m3 rows (uint8 tensors; ``dtype_code`` must be
    ``RB_E4M3``, scales ``None``): the score is the fp32 accumulator (exact for
    ±1 codes). C-ABI ``rb_dense_topk_scaled``."""
    if queries.dim() != 2 or items.dim() != 2 or queries.shape[1] != items.shape[1]:
        raise ValueError("queries [B, D] and items [N, D] with the same D")
    _require_cuda(queries, items)
    check_contiguous(items=items)
    q = queries.contiguous()
    b, d = q.shape
    n = items.shape[0]
    dev = q.device
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    qs = None if query_scales is None else query_scales.to(torch.float32).contiguous()
    xs = None if item_scales is None else item_scales.to(torch.float32).contiguous()
    lib = _lib.lib()
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_workspace_size(b, n, d, dtype_code, k, ctypes.byref(nb)), "scaled_topk")
    ws = torch.empty(max(int(nb.value), 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.rb_dense_topk_scaled(_ptr(q), _ptr(qs), _ptr(items), _ptr(xs), b, n, d, dtype_code, k,
                                      int(id_offset), _ptr(ids), _ptr(scores), _ptr(ws), ws.numel(), _stream_ptr(dev))
    _lib.check(rc, "scaled_topk")
    return ids, scores


def int8_codes_topk(
    query_codes: Tensor, query_scales: Tensor | None, item_codes: Tensor, item_scales: Tensor | None, k: int,
    id_offset: int = 0,
) -> tuple[Tensor, Tensor]:
    """Tensor-core int8 scoring of already-quantized queries (C-ABI
    ``rb_dense_topk_i8``): score ``(fp32(dot) * query_scale) * item_scale``; a
    ``None`` scale means 1 (the score is then the exact int32 dot)."""
    if query_codes.dtype != torch.int8 or item_codes.dtype != torch.int8:
        raise TypeError("query_codes and item_codes must be int8")
    if query_codes.dim() != 2 or item_codes.dim() != 2 or query_codes.shape[1] != item_codes.shape[1]:
        raise ValueError("query_codes [B, D] and item_codes [N, D] with the same D")
    _require_cuda(query_codes, item_codes)
    check_contiguous(item_codes=item_codes)
    codes = query_codes.contiguous()
    b, d = codes.shape
    n = item_codes.shape[0]
    dev = codes.device
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    qs = None if query_scales is None else query_scales.to(torch.float32).contiguous()
    xs = None if item_scales is None else item_scales.to(torch.float32).contiguous()
    lib = _lib.lib()
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_workspace_size(b, n, d, _lib.RB_I8, k, ctypes.byref(nb)), "int8_topk")
    ws = torch.empty(max(int(nb.value), 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.rb_dense_topk_i8(_ptr(codes), _ptr(qs), _ptr(item_codes), _ptr(xs), b, n, d, k, int(id_offset),
                                  _ptr(ids), _ptr(scores), _ptr(ws), ws.numel(), _stream_ptr(dev))
    _lib.check(rc, "int8_topk")
    return ids, scores


def bits_to_pm1(bits: Tensor, fmt: str = "int8") -> Tensor:
    """1-bit codes ``[N, W]`` int64 → ``[N, 64 W]`` rows of ±1 (+1 where the bit
    is set): int8 (C-ABI ``rb_bits_to_pm1``) or fp8 e4m3 bytes as uint8
    (``fmt="e4m3"``, ``rb_bits_to_pm1_e4m3``). The dot of two such rows is the
    1-bit match score ``64 W − 2·popcount(q ^ x)``."""
    if bits.dim() != 2 or bits.dtype != torch.int64:
        raise ValueError("bits must be [N, W] int64")
    if fmt not in ("int8", "e4m3"):
        raise ValueError(f"fmt must be 'int8' or 'e4m3', got {fmt!r}")
    _require_cuda(bits)
    bits = bits.contiguous()
    n, w = bits.shape
    e4m3 = fmt == "e4m3"
    out = torch.empty((n, 64 * w), dtype=torch.uint8 if e4m3 else torch.int8, device=bits.device)
    if n == 0:
        return out
    fn = _lib.lib().rb_bits_to_pm1_e4m3 if e4m3 else _lib.lib().rb_bits_to_pm1
    with torch.cuda.device(bits.device):
        rc = fn(_ptr(bits), n, w, _ptr(out), _stream_ptr(bits.device))
    _lib.check(rc, "bits_to_pm1")
    return out


@int8_topk.register_fake
def _(query, item_codes, item_scales, k):
    b = query.shape[0]
    return query.new_empty((b, k), dtype=torch.int64), query.new_empty((b, k), dtype=torch.float32)


__all__ = [
    "bits_to_pm1",
    "bloom_build",
    "dense_topk_filtered",
    "check_contiguous",
    "int8_topk",
    "int8_codes_topk",
    "scaled_topk",
    "clause_compact",
    "clause_mask",
    "clause_mask_scores",
    "dense_topk",
    "dense_topk_sharded",
    "fused_masked_knn_topk",
    "gemv_scores",
    "oporp_1bit_match_topk_full",
    "oporp_1bit_match_topk_indirect",
    "quantize_int8",
]
