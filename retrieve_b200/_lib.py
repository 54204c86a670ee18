"""ctypes binding of ``libretrieve_b200.so`` (the C-ABI declared in
``include/retrieve_b200.h``).

The library is built in-tree by ``retrieve_b200.build``; there is no fallback:
if it is missing or fails to load, :func:`lib` raises ``ImportError`` naming
the cause, so no op can silently run on another implementation.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libretrieve_b200.so"
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "retrieve_b200.h"

RB_OK = 0
RB_ERR_INVALID_ARG = 1
RB_ERR_TYPE = 2
RB_ERR_UNSUPPORTED = 3
RB_ERR_WORKSPACE = 4
RB_ERR_CUDA = 5
RB_ERR_DEVICE = 6

RB_F16, RB_BF16, RB_I8, RB_F32, RB_E4M3 = 0, 1, 2, 3, 4

_c_int = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p

class StFilter(ctypes.Structure):
    """``rb_st_filter`` of include/retrieve_b200.h: at most one of the three filters."""

    _fields_ = [
        ("filtering_bit_mask", _vp), ("mask_words", _c_i64),
        ("item_clause_attrs", _vp), ("attr_rows", _c_i64), ("attr_docs", _c_i64), ("clause_slots", _vp),
        ("clause_is_reverse", _vp), ("query_clause_attrs", _vp), ("n_clauses", _c_int),
        ("bloom_index", _vp), ("bloom_words", _c_i64), ("bundle_b_offsets", _vp), ("n_bundles", _c_i64),
        ("plans", _vp), ("plan_words", _c_i64), ("plan_count", _c_int), ("max_stack_size", _c_int),
        ("query_plan_index", _vp), ("bloom_k", _c_int), ("hash_k", _c_int),
    ]  # fmt: skip


# name -> (restype, argtypes); mirrors include/retrieve_b200.h
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "rb_last_error": (ctypes.c_char_p, []),
    "rb_abi_version": (_c_int, []),
    "rb_dense_topk_workspace_size": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_dense_topk": (
        _c_int,
        [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _vp, _vp, _vp, _c_size, _vp],
    ),
    "rb_dense_topk_filtered_workspace_size": (
        _c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]
    ),
    "rb_dense_topk_filtered": (
        _c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _vp, _vp, _vp, _vp, _c_size, _vp]
    ),
    "rb_bloom_build": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "rb_bloom_slices_bytes": (_c_int, [_c_i64, ctypes.POINTER(_c_size)]),
    "rb_bloom_slices": (_c_int, [_vp, _c_i64, _vp, _vp]),
    "rb_dense_topk_i8": (
        _c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_i64, _vp, _vp, _vp, _c_size, _vp]
    ),
    "rb_dense_topk_launches": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_int)]),
    "rb_merge_topk_workspace_size": (_c_int, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_merge_topk": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_size, _vp]),
    "rb_set_profile_events": (_c_int, [_vp, _vp]),
    "rb_workspace_device_error": (_c_int, [_vp, _c_size, ctypes.POINTER(_c_int)]),
    "rb_wait_probe": (_c_int, [_c_i64, _vp, _c_size, _vp]),
    "rb_dense_seed_sample": (
        _c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _vp, _vp, _c_size, _vp]
    ),
    "rb_dense_topk_seeded": (
        _c_int,
        [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_i64, _vp, _c_int, _c_int, _vp, _vp, _vp, _vp,
         _c_size, _vp],
    ),
    "rb_merge_pairs": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp]),
    "rb_ipc_alloc": (_c_int, [_c_size, ctypes.POINTER(_vp), _vp]),
    "rb_ipc_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "rb_ipc_close": (_c_int, [_vp]),
    "rb_ipc_free": (_c_int, [_vp]),
    "rb_peer_buffer_bytes": (_c_size, [_c_int, _c_i64]),
    "rb_peer_allgather": (
        _c_int, [ctypes.POINTER(_vp), _c_int, _c_int, _c_i64, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp]
    ),
    "rb_quantize_int8_global_workspace_size": (_c_int, [ctypes.POINTER(_c_size)]),
    "rb_quantize_int8_global": (_c_int, [_vp, _c_i64, _c_int, _vp, _c_i64, _vp, _vp, _vp, _c_size, _vp]),
    "rb_pack_signs": (_c_int, [_vp, _c_i64, _c_int, _vp, _vp]),
    "rb_bloom_index_widths": (_c_int, [_vp, _c_i64, _c_int, _c_int, ctypes.c_double, _c_i64, _vp, _vp, _vp]),
    "rb_bloom_index_fill": (_c_int, [_vp, _vp, _vp, _c_i64, _c_i64, _c_int, _c_int, _vp, _vp, _c_i64, _vp]),
    "rb_st_search_workspace_size": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_st_search": (
        _c_int,
        [_vp, _c_int, _c_int, _vp, _c_int, _vp, _vp, _c_i64, _vp, _c_i64, _vp, _vp, _c_int, _c_int, _c_int,
         ctypes.POINTER(StFilter), _vp, _vp, _vp, _c_size, _vp],
    ),
    "rb_st_search_grouped_workspace_size": (
        _c_int, [_c_int, _c_int, _c_int, _c_i64, _c_int, _c_int, ctypes.POINTER(_c_size)]
    ),
    "rb_st_search_grouped": (
        _c_int,
        [_vp, _c_int, _c_int, _vp, _c_int, _vp, _vp, _c_i64, _vp, _c_i64, _vp, _vp, _c_int, _c_int, _c_int,
         ctypes.POINTER(StFilter), _vp, _vp, _vp, _c_size, _vp],
    ),
    "rb_st_search_shard": (
        _c_int,
        [_vp, _c_int, _c_int, _vp, _c_int, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _c_int, _c_int, _c_int,
         ctypes.POINTER(StFilter), _vp, _vp, _c_size, _vp],
    ),
    "rb_st_search_finish_workspace_size": (_c_int, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_st_search_finish": (
        _c_int,
        [_vp, _c_int, _c_int, _vp, _c_int, _vp, _vp, _c_i64, _c_i64, _vp, _vp, _c_int, _c_int, _c_int, _vp, _vp,
         _c_int, _vp, _vp, _vp, _c_size, _vp],
    ),
    "rb_st_fused_kmean_ann_workspace_size": (_c_int, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_st_fused_kmean_ann": (
        _c_int,
        [_vp, _c_i64, _vp, _vp, _c_int, _vp, _c_i64, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _c_i64, _c_i64, _vp,
         _vp, _c_int, _c_int, _vp, _vp, _vp, _c_size, _vp],
    ),
    "rb_st_fused_kmean_ann_with_partial_masks": (
        _c_int,
        [_vp, _c_i64, _vp, _vp, _c_int, _vp, _c_i64, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_i64,
         _c_i64, _vp, _vp, _c_int, _c_int, _vp, _vp, _vp, _c_size, _vp],
    ),
    "rb_st_bloom_search": (
        _c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp]
    ),
    "rb_st_bloom_column_info": (_c_int, [_vp, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp]),
    "rb_st_bloom_partial_search": (
        _c_int,
        [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp, _c_int, _c_int, _vp,
         _c_i64, _vp],
    ),
    "rb_st_fresh_topk": (_c_int, [_vp, _c_i64, _vp, _c_i64, _c_int, _c_i64, _c_int, _vp, _vp, _vp, _vp]),
    "rb_st_fresh_gather": (
        _c_int,
        [_vp, _c_i64, _c_int, _c_i64, _c_i64, _vp, _vp, _c_int, _vp, _c_i64, _vp, _c_i64, _c_i64, _c_int, _vp, _vp],
    ),
    "rb_st_is_topk": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _vp, _c_int, _vp, _vp]),
    "rb_kmeans_cluster_sums_workspace_size": (_c_int, [_c_i64, _c_i64, ctypes.POINTER(_c_size)]),
    "rb_kmeans_cluster_sums": (
        _c_int, [_vp, _c_int, _c_i64, _c_int, _vp, _c_i64, _vp, _vp, _vp, _c_size, _vp]
    ),
    "rb_st_parse_expression_batch": (
        _c_int, [_vp, _vp, _c_int, _c_i64, _c_i64, _vp, _c_i64, _vp, _vp, _vp]
    ),
    "rb_st_probe_prep": (
        _c_int,
        [_vp, _c_int, _c_int, _vp, _c_int, _vp, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "rb_bits_to_pm1": (_c_int, [_vp, _c_int, _c_int, _vp, _vp]),
    "rb_bits_to_pm1_e4m3": (_c_int, [_vp, _c_int, _c_int, _vp, _vp]),
    "rb_dense_topk_scaled": (
        _c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _vp, _vp, _vp, _c_size, _vp]
    ),
    "rb_clause_mask": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _c_int, _vp, _vp, _vp]),
    "rb_clause_compact_workspace_size": (_c_int, [_c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_clause_compact": (
        _c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _c_int, _vp, _vp, _vp, _c_size, _vp]
    ),
    "rb_gemv_scores": (_c_int, [_vp, _vp, _c_int, _c_int, _vp, _vp]),
    "rb_candidate_topk_workspace_size": (_c_int, [_c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_candidate_topk": (
        _c_int,
        [_c_int, _vp, _c_int, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _vp, _c_int, _c_int, _vp, _vp, _vp,
         _c_size, _vp],
    ),
    "rb_hamming_topk_workspace_size": (_c_int, [_c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "rb_hamming_topk": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_size, _vp]),
    "rb_quantize_int8": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _vp]),
    "rb_dense_topk_noalloc_scratch_bytes": (_c_size, []),
    "rb_dense_topk_noalloc": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _vp, _vp, _vp]),
}

_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once). Raises ``ImportError`` if it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python -m retrieve_b200.build` "
            "(the CUDA kernels are the only implementation of these ops)"
        )
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = handle
    return handle


def header_symbols() -> list[str]:
    """Every function the public header declares (``RB_API`` prototypes)."""
    text = HEADER_PATH.read_text()
    return re.findall(r"^RB_API\s+[\w\s\*]+?\b(rb_\w+)\s*\(", text, flags=re.M)


def check(rc: int, what: str) -> None:
    """Maps a C-ABI status to the reference's Python exception convention."""
    if rc == RB_OK:
        return
    msg = lib().rb_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if msg else what
    if rc == RB_ERR_INVALID_ARG or rc == RB_ERR_UNSUPPORTED:
        raise ValueError(text)
    if rc == RB_ERR_TYPE:
        raise TypeError(text)
    raise RuntimeError(f"{text} (status {rc})")
