"""The ``torch.ops.st`` namespace on ``libretrieve_b200.so``.

SilverTorch's one-op IVF forward ``st::search`` and its prep ``st::probe_prep``
(silvertorch/ops/csrc/fork_search.cpp:13-49, fork_search_cuda.cu:1256-1546), reached
by the reference through ``adapter.fork_search``
(retrieve/src/retrieve/ops/official/adapter.py:495-544), and the upstream-shaped ops
of the reference's loader list around it: the raw scorers ``st::fused_kmean_ann`` and
``st::fused_kmean_ann_with_partial_masks`` (int8 codes), the bloom index builds, the
bloom searches and the expression parser (``retrieve_b200.st_bloom``). Importing this
module registers their implementations under the reference's exact schemas: it defines
a schema when no other library has, and otherwise adds the CUDA kernels to the
definitions already loaded (the reference's CPU build keeps serving the CPU key).

Semantics: int8 query prep as ``quantize_int8`` on a CUDA tensor, the probed
clusters' positions in the reference scorer's slot order, exact int32 dots,
top-k on the raw score with ties to the lower slot, ``id = sort_perm[pos]`` and
``score = (fp32(dot) * q_scale) * global_scale`` (or the fp16 path's
``raw * ((q_scale * divisor) * global_scale)``), ``-1`` / ``-inf`` pads. A
full-``N`` ``filtering_bit_mask`` (high bit first), the exact clause filter and
SilverTorch's bloom over its own index and prepared plans are served; bloom plans
with the exact recheck give the exact filter's result (the bloom has no false
negatives), so the plans are then not read.
Errors raise ``RuntimeError``, as the reference's ``TORCH_CHECK``s do.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from retrieve_b200 import _lib, st_bloom, st_select
from retrieve_b200._st_common import _call, _check, _ptr, _stream

SEARCH_SCHEMA = (
    "search(Tensor query, Tensor probe_ids, Tensor cluster_offsets, Tensor cluster_sizes, "
    "Tensor item_codes, Tensor sort_perm, Tensor global_scale, int k, int max_tensor_size_per_row, "
    "int divisor_for_int8=-1, Tensor? filtering_bit_mask=None, Tensor? bloom_index=None, "
    "Tensor? bloom_bundle_b_offsets=None, Tensor? plans=None, int plan_count=0, int max_stack_size=0, "
    "Tensor? query_plan_index=None, int bloom_k=0, int hash_k=0, Tensor? item_clause_attrs=None, "
    "Tensor? clause_slots=None, Tensor? clause_is_reverse=None, Tensor? query_clause_attrs=None) "
    "-> (Tensor, Tensor)"
)
PROBE_PREP_SCHEMA = (
    "probe_prep(Tensor query, Tensor probe_ids, Tensor cluster_offsets, Tensor cluster_sizes) "
    "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)"
)


def _layout_args(query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor):
    _check(query.dim() == 2, "query must be [B, D]")
    _check(probe_ids.dim() == 2 and probe_ids.shape[0] == query.shape[0], "probe_ids must be [B, n_probe]")
    _check(cluster_offsets.dim() == 1 and cluster_sizes.dim() == 1, "cluster_offsets / cluster_sizes must be 1-D")
    for name, t in (("query", query), ("probe_ids", probe_ids), ("cluster_offsets", cluster_offsets),
                    ("cluster_sizes", cluster_sizes)):
        _check(t.is_cuda, f"st ops run on CUDA tensors only ({name} is on {t.device})")
    q = query.to(torch.float32).contiguous()
    probe = probe_ids.to(torch.int64).contiguous()
    offsets = cluster_offsets.to(torch.int64).contiguous()
    sizes = cluster_sizes.to(torch.int64).contiguous()
    return q, probe, offsets, sizes


# The schema's filter arguments, in schema order (fork_search.cpp:24-37). The dispatcher
# passes every argument up to the last one given positionally, as the reference's
# adapter.fork_search does (adapter.py:522-544), so the impls name each one.
FILTER_ARGS = ("filtering_bit_mask", "bloom_index", "bloom_bundle_b_offsets", "plans", "plan_count",
               "max_stack_size", "query_plan_index", "bloom_k", "hash_k", "item_clause_attrs", "clause_slots",
               "clause_is_reverse", "query_clause_attrs")


def search(query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor, item_codes: Tensor,
           sort_perm: Tensor, global_scale: Tensor, k: int, max_tensor_size_per_row: int, divisor_for_int8: int = -1,
           filtering_bit_mask: Tensor | None = None, bloom_index: Tensor | None = None,
           bloom_bundle_b_offsets: Tensor | None = None, plans: Tensor | None = None, plan_count: int = 0,
           max_stack_size: int = 0, query_plan_index: Tensor | None = None, bloom_k: int = 0, hash_k: int = 0,
           item_clause_attrs: Tensor | None = None, clause_slots: Tensor | None = None,
           clause_is_reverse: Tensor | None = None,
           query_clause_attrs: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """``st::search`` → ``(ids int64 [B, k], scores fp32 [B, k])``. Takes the schema's 23
    arguments positionally or by name. Scored by cluster (``search_grouped``: each probed
    cluster read once per group of probing rows) up to 1024 probes a row unless bloom plans
    are given without the exact recheck; else row by row (each row's probed positions
    expanded, then the int8 candidate scan), where the bloom plans are evaluated once per
    64-doc column. Both give the same results."""
    filters = dict(zip(FILTER_ARGS, (filtering_bit_mask, bloom_index, bloom_bundle_b_offsets, plans, plan_count,
                                     max_stack_size, query_plan_index, bloom_k, hash_k, item_clause_attrs,
                                     clause_slots, clause_is_reverse, query_clause_attrs)))
    bloom_only = plans is not None and query_clause_attrs is None
    grouped = not bloom_only and probe_ids.dim() == 2 and probe_ids.shape[1] <= 1024
    return _search(grouped, query, probe_ids, cluster_offsets, cluster_sizes, item_codes, sort_perm, global_scale, k,
                   max_tensor_size_per_row, divisor_for_int8, filters)


def search_rows(query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor,
                item_codes: Tensor, sort_perm: Tensor, global_scale: Tensor, k: int, max_tensor_size_per_row: int,
                divisor_for_int8: int = -1, filtering_bit_mask: Tensor | None = None,
                bloom_index: Tensor | None = None, bloom_bundle_b_offsets: Tensor | None = None,
                plans: Tensor | None = None, plan_count: int = 0, max_stack_size: int = 0,
                query_plan_index: Tensor | None = None, bloom_k: int = 0, hash_k: int = 0,
                item_clause_attrs: Tensor | None = None, clause_slots: Tensor | None = None,
                clause_is_reverse: Tensor | None = None,
                query_clause_attrs: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """``st::search`` scored row by row (``rb_st_search``) whatever the filter: the same
    arguments and results as ``search``."""
    filters = dict(zip(FILTER_ARGS, (filtering_bit_mask, bloom_index, bloom_bundle_b_offsets, plans, plan_count,
                                     max_stack_size, query_plan_index, bloom_k, hash_k, item_clause_attrs,
                                     clause_slots, clause_is_reverse, query_clause_attrs)))
    return _search(False, query, probe_ids, cluster_offsets, cluster_sizes, item_codes, sort_perm, global_scale, k,
                   max_tensor_size_per_row, divisor_for_int8, filters)


def search_grouped(query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor,
                   item_codes: Tensor, sort_perm: Tensor, global_scale: Tensor, k: int, max_tensor_size_per_row: int,
                   divisor_for_int8: int = -1, filtering_bit_mask: Tensor | None = None,
                   bloom_index: Tensor | None = None, bloom_bundle_b_offsets: Tensor | None = None,
                   plans: Tensor | None = None, plan_count: int = 0, max_stack_size: int = 0,
                   query_plan_index: Tensor | None = None, bloom_k: int = 0, hash_k: int = 0,
                   item_clause_attrs: Tensor | None = None, clause_slots: Tensor | None = None,
                   clause_is_reverse: Tensor | None = None,
                   query_clause_attrs: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """``st::search`` with the scoring grouped by cluster (``rb_st_search_grouped``): the
    same arguments and results; each probed cluster is read once per group of up to 64
    probing rows. Up to 1024 probes a row."""
    filters = dict(zip(FILTER_ARGS, (filtering_bit_mask, bloom_index, bloom_bundle_b_offsets, plans, plan_count,
                                     max_stack_size, query_plan_index, bloom_k, hash_k, item_clause_attrs,
                                     clause_slots, clause_is_reverse, query_clause_attrs)))
    return _search(True, query, probe_ids, cluster_offsets, cluster_sizes, item_codes, sort_perm, global_scale, k,
                   max_tensor_size_per_row, divisor_for_int8, filters)


_FILTER_DOC = """Filters: a full-``N`` ``filtering_bit_mask``; the exact clauses
    (``item_clause_attrs``, ``clause_slots``, ``clause_is_reverse``, ``query_clause_attrs``);
    or SilverTorch's bloom (``bloom_index``, ``bloom_bundle_b_offsets``, the prepared ``plans``
    blob of ``plan_count`` slots, ``max_stack_size``, ``query_plan_index``, ``bloom_k``,
    ``hash_k``), false positives kept. With bloom plans and the exact clauses together (the
    bloom with its exact recheck) the result is the exact filter's, since the bloom has no
    false negatives; the plans are then not read."""


def _filter(query: Tensor, n_items: int, filtering_bit_mask=None, bloom_index=None, bloom_bundle_b_offsets=None,
            plans=None, plan_count=0, max_stack_size=0, query_plan_index=None, bloom_k=0, hash_k=0,
            item_clause_attrs=None, clause_slots=None, clause_is_reverse=None, query_clause_attrs=None):
    """The call's ``rb_st_filter`` (or None) and the tensors it points into."""
    exact = query_clause_attrs is not None
    _check(not (filtering_bit_mask is not None and (plans is not None or exact)),
           "search takes one filter: plans (+ query_clause_attrs to recheck), query_clause_attrs or "
           "filtering_bit_mask")
    flt = _lib.StFilter()
    keep: list[Tensor] = []
    if exact:
        _check(item_clause_attrs is not None and clause_slots is not None and clause_is_reverse is not None,
               "the exact filter needs item_clause_attrs, clause_slots and clause_is_reverse")
        _check(item_clause_attrs.dim() == 2 and item_clause_attrs.dtype == torch.int32,
               "item_clause_attrs must be int32 [R, N]")
        _check(clause_slots.dim() == 1 and clause_slots.dtype == torch.int64, "clause_slots must be int64 [C + 1]")
        _check(query_clause_attrs.dim() == 2 and query_clause_attrs.dtype == torch.int32,
               "query_clause_attrs must be int32 [B, C]")
        _check(clause_is_reverse.dtype == torch.bool, "clause_is_reverse must be bool")
        for t in (item_clause_attrs, clause_slots, clause_is_reverse, query_clause_attrs):
            _check(t.is_contiguous() and t.device == query.device,
                   "the exact filter's tensors must be contiguous and on the query's device")
        n_clauses = query_clause_attrs.shape[1]
        _check(clause_slots.shape[0] == n_clauses + 1 and clause_is_reverse.numel() == n_clauses,
               "clause_slots must have C + 1 entries and clause_is_reverse C")
        _check(query_clause_attrs.shape[0] == query.shape[0], "query_clause_attrs must have B rows")
        _check(item_clause_attrs.shape[1] >= n_items, "item_clause_attrs must cover the N docs")
        flt.item_clause_attrs = item_clause_attrs.data_ptr()
        flt.attr_rows, flt.attr_docs = item_clause_attrs.shape
        flt.clause_slots = clause_slots.data_ptr()
        flt.clause_is_reverse = clause_is_reverse.data_ptr()
        flt.query_clause_attrs = query_clause_attrs.data_ptr()
        flt.n_clauses = n_clauses
        return flt, keep
    if plans is not None:
        _check(bloom_index is not None and bloom_bundle_b_offsets is not None,
               "the bloom filter needs bloom_index and bloom_bundle_b_offsets")
        for name, t in (("bloom_index", bloom_index), ("bloom_bundle_b_offsets", bloom_bundle_b_offsets),
                        ("plans", plans)):
            _check(t.dtype == torch.int64 and t.dim() == 1 and t.is_contiguous() and t.device == query.device,
                   f"{name} must be a contiguous 1-D int64 tensor on the query's device")
        _check(plan_count >= 1 and plans.numel() >= 8 * plan_count, "plans must hold plan_count slots")
        if query_plan_index is not None:
            _check(query_plan_index.dtype == torch.int64 and query_plan_index.numel() == query.shape[0]
                   and query_plan_index.is_contiguous() and query_plan_index.device == query.device,
                   "query_plan_index must be int64 [B] on the query's device")
        else:
            _check(plan_count >= query.shape[0], "without query_plan_index every row needs its own plan")
        flt.bloom_index = bloom_index.data_ptr()
        flt.bloom_words = bloom_index.numel()
        flt.bundle_b_offsets = bloom_bundle_b_offsets.data_ptr()
        flt.n_bundles = bloom_bundle_b_offsets.numel() - 1
        flt.plans = plans.data_ptr()
        flt.plan_words = plans.numel()
        flt.plan_count = int(plan_count)
        flt.max_stack_size = int(max_stack_size)
        flt.query_plan_index = 0 if query_plan_index is None else query_plan_index.data_ptr()
        flt.bloom_k = int(bloom_k)
        flt.hash_k = int(hash_k)
        return flt, keep
    if filtering_bit_mask is not None:
        _check(filtering_bit_mask.dim() == 2 and filtering_bit_mask.shape[0] == query.shape[0],
               "filtering_bit_mask must be [B, words]")
        mask = filtering_bit_mask.to(device=query.device, dtype=torch.int64).contiguous()
        keep.append(mask)
        flt.filtering_bit_mask = mask.data_ptr()
        flt.mask_words = mask.shape[1]
        return flt, keep
    return None, keep


def _codes_check(item_codes: Tensor, query: Tensor) -> None:
    """The reference's first check (fork_search_cuda.cu:1280), before any device check."""
    _check(item_codes.dtype == torch.int8 and item_codes.dim() == 2 and item_codes.shape[1] == query.shape[1],
           "item_codes must be int8 [N, D] with the query's D")
    _check(item_codes.is_contiguous(), "item_codes must be contiguous")


def _search(
    grouped: bool,
    query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor, item_codes: Tensor,
    sort_perm: Tensor, global_scale: Tensor, k: int, max_tensor_size_per_row: int, divisor_for_int8: int,
    filters: dict,
) -> tuple[Tensor, Tensor]:
    _codes_check(item_codes, query)
    flt, keep = _filter(query, item_codes.shape[0], **filters)
    q, probe, offsets, sizes = _layout_args(query, probe_ids, cluster_offsets, cluster_sizes)
    _check(item_codes.device == q.device, "item_codes must be on the query's device")
    _check(offsets.numel() == sizes.numel() + 1, "cluster_offsets must have n_lists + 1 entries")
    _check(sort_perm.dim() == 1 and sort_perm.numel() == item_codes.shape[0], "sort_perm must be [N]")
    dev = q.device
    perm = sort_perm.to(device=dev, dtype=torch.int64).contiguous()
    gs = global_scale.to(device=dev, dtype=torch.float32).reshape(-1)[:1].contiguous()
    _check(gs.numel() == 1, "global_scale must hold one value")
    b, d = q.shape
    p = probe.shape[1]
    _check(k >= 1, f"k must be positive, got {k}")
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    if grouped:
        _call(lib.rb_st_search_grouped_workspace_size(b, d, p, sizes.numel(), k, int(max_tensor_size_per_row),
                                                      ctypes.byref(nbytes)), "st::search")
    else:
        _call(lib.rb_st_search_workspace_size(b, d, p, k, int(max_tensor_size_per_row), ctypes.byref(nbytes)),
              "st::search")
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
    rc = (lib.rb_st_search_grouped if grouped else lib.rb_st_search)(
        _ptr(q), b, d, _ptr(probe), p, _ptr(offsets), _ptr(sizes), sizes.numel(), _ptr(item_codes),
        item_codes.shape[0], _ptr(perm), _ptr(gs), k, int(max_tensor_size_per_row), int(divisor_for_int8),
        ctypes.byref(flt) if flt is not None else None, _ptr(ids), _ptr(scores), _ptr(ws), ws.numel(), _stream(dev),
    )
    _call(rc, "st::search")
    del keep
    return ids, scores


_search.__doc__ = _FILTER_DOC


def search_shard(query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor, n_total: int,
                 pos_lo: int, item_codes: Tensor, k: int, max_tensor_size_per_row: int, divisor_for_int8: int = -1,
                 **filters) -> Tensor:
    """One rank's part of a row-sharded ``st::search`` (``rb_st_search_shard``): the table's
    rows ``[pos_lo, pos_lo + len(item_codes))`` scored in the whole table's slot layout →
    packed ``(raw score bits, slot)`` pairs ``[B, min(k, width)]`` int64 for ``ops.merge_pairs``.
    The probe tables and the filter are the whole table's."""
    _codes_check(item_codes, query)
    flt, keep = _filter(query, int(n_total), **filters)
    q, probe, offsets, sizes = _layout_args(query, probe_ids, cluster_offsets, cluster_sizes)
    _check(item_codes.device == q.device, "item_codes must be on the query's device")
    b, d = q.shape
    p = probe.shape[1]
    _check(k >= 1, f"k must be positive, got {k}")
    width = (int(max_tensor_size_per_row) + 31) // 32 * 32
    pairs = torch.empty((b, min(k, width)), dtype=torch.int64, device=q.device)
    if b == 0:
        return pairs
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _call(lib.rb_st_search_workspace_size(b, d, p, k, int(max_tensor_size_per_row), ctypes.byref(nbytes)),
          "st::search shard")
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=q.device)
    rc = lib.rb_st_search_shard(
        _ptr(q), b, d, _ptr(probe), p, _ptr(offsets), _ptr(sizes), sizes.numel(), int(n_total), int(pos_lo),
        int(pos_lo) + item_codes.shape[0], _ptr(item_codes), k, int(max_tensor_size_per_row), int(divisor_for_int8),
        ctypes.byref(flt) if flt is not None else None, _ptr(pairs), _ptr(ws), ws.numel(), _stream(q.device),
    )
    _call(rc, "st::search shard")
    del keep
    return pairs


def search_finish(query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor,
                  sort_perm: Tensor, global_scale: Tensor, k: int, max_tensor_size_per_row: int, slots: Tensor,
                  raw: Tensor, divisor_for_int8: int = -1) -> tuple[Tensor, Tensor]:
    """Merged ``(slots, raw)`` ``[B, kin]`` of a row-sharded search → ``(ids [B, k], scores
    [B, k])`` through the whole table's layout (``rb_st_search_finish``)."""
    q, probe, offsets, sizes = _layout_args(query, probe_ids, cluster_offsets, cluster_sizes)
    dev = q.device
    b, d = q.shape
    p = probe.shape[1]
    perm = sort_perm.to(device=dev, dtype=torch.int64).contiguous()
    gs = global_scale.to(device=dev, dtype=torch.float32).reshape(-1)[:1].contiguous()
    sl = slots.to(device=dev, dtype=torch.int64).contiguous()
    rw = raw.to(device=dev, dtype=torch.float32).contiguous()
    _check(sl.shape == rw.shape and sl.dim() == 2 and sl.shape[0] == b, "slots and raw must both be [B, kin]")
    ids = torch.empty((b, k), dtype=torch.int64, device=dev)
    scores = torch.empty((b, k), dtype=torch.float32, device=dev)
    if b == 0:
        return ids, scores
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _call(lib.rb_st_search_finish_workspace_size(b, d, p, ctypes.byref(nbytes)), "st::search finish")
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
    rc = lib.rb_st_search_finish(
        _ptr(q), b, d, _ptr(probe), p, _ptr(offsets), _ptr(sizes), sizes.numel(), perm.numel(), _ptr(perm), _ptr(gs),
        k, int(max_tensor_size_per_row), int(divisor_for_int8), _ptr(sl), _ptr(rw), sl.shape[1], _ptr(ids),
        _ptr(scores), _ptr(ws), ws.numel(), _stream(dev),
    )
    _call(rc, "st::search finish")
    return ids, scores


def probe_prep(query: Tensor, probe_ids: Tensor, cluster_offsets: Tensor, cluster_sizes: Tensor):
    """``st::probe_prep`` → its nine layout tensors (fork_search.cpp:43-49)."""
    q, probe, offsets, sizes = _layout_args(query, probe_ids, cluster_offsets, cluster_sizes)
    b, d = q.shape
    p = probe.shape[1]
    dev = q.device
    codes = torch.empty((b, d), dtype=torch.int8, device=dev)
    scales = torch.empty((b,), dtype=torch.float32, device=dev)
    cids = torch.empty((b, p), dtype=torch.int64, device=dev)
    length = torch.empty((b, p), dtype=torch.int64, device=dev)
    offs = torch.empty((b, p), dtype=torch.int64, device=dev)
    warps = torch.empty((b * p,), dtype=torch.int32, device=dev)
    rounded = torch.empty((b, p), dtype=torch.int32, device=dev)
    rem = torch.empty((b * p,), dtype=torch.int32, device=dev)
    wcum = torch.empty((b * p,), dtype=torch.int32, device=dev)
    if b > 0:
        rc = _lib.lib().rb_st_probe_prep(
            _ptr(q), b, d, _ptr(probe), p, _ptr(offsets), _ptr(sizes), sizes.numel(), _ptr(codes), _ptr(scales),
            _ptr(cids), _ptr(length), _ptr(offs), _ptr(warps), _ptr(rounded), _ptr(rem), _ptr(wcum), _stream(dev),
        )
        _call(rc, "st::probe_prep")
    return codes, scales, cids, length, offs, warps, rounded, rem, wcum


BLOOM_BUILD_SCHEMA = (
    "bloom_index_build(Tensor feature_ids, Tensor feature_offsets, Tensor feature_values, "
    "float b_multiplier, int k, bool fast_build=False) -> (Tensor, Tensor)"
)
BLOOM_BUILD_FIXED_SCHEMA = (
    "bloom_index_build_fixed(Tensor feature_ids, Tensor feature_offsets, Tensor feature_values, "
    "int bits_per_doc, int k, bool fast_build=False) -> (Tensor, Tensor)"
)


def _bloom_build(feature_ids: Tensor, feature_offsets: Tensor, feature_values: Tensor, b_multiplier: float,
                 bits_per_doc: int, k: int) -> tuple[Tensor, Tensor]:
    _check(feature_ids.dtype == torch.int32 and feature_offsets.dtype == torch.int64
           and feature_values.dtype == torch.int64, "feature_ids int32, feature_offsets and feature_values int64")
    for t in (feature_ids, feature_offsets, feature_values):
        _check(t.is_cuda and t.dim() == 1, "the bloom build takes 1-D CUDA tensors")
    c = feature_ids.numel()
    _check(c > 0 and (feature_offsets.numel() - 1) % c == 0, "feature_offsets must have N * C + 1 entries")
    if bits_per_doc <= 0:
        _check(b_multiplier > 1.0, "b_multiplier must be greater than 1.0")
    dev = feature_ids.device
    fid, foff, fval = (t.contiguous() for t in (feature_ids, feature_offsets, feature_values))
    n = (foff.numel() - 1) // c
    n_bundles = (n + 2047) // 2048
    widths = torch.empty(max(n_bundles, 1), dtype=torch.int64, device=dev)
    offsets = torch.empty(n_bundles + 1, dtype=torch.int64, device=dev)
    lib = _lib.lib()
    _call(lib.rb_bloom_index_widths(_ptr(foff), n, c, int(k), float(b_multiplier), int(bits_per_doc), _ptr(widths),
                                    _ptr(offsets), _stream(dev)), "bloom_index_build")
    words = int(offsets[-1].item()) * 32  # the index size: one host read, as the reference's builders
    index = torch.zeros(words, dtype=torch.int64, device=dev)
    _call(lib.rb_bloom_index_fill(_ptr(fid), _ptr(foff), _ptr(fval), fval.numel(), n, c, int(k), _ptr(offsets),
                                  _ptr(index), words, _stream(dev)), "bloom_index_build")
    return index, offsets


def bloom_index_build(feature_ids: Tensor, feature_offsets: Tensor, feature_values: Tensor, b_multiplier: float,
                      k: int, fast_build: bool = False) -> tuple[Tensor, Tensor]:
    """``st::bloom_index_build`` on the device: ``(bloom_index int64, bundle_b_offsets int64)``,
    each 2048-doc bundle ``trunc(max values a doc * k * b_multiplier)`` bits per doc.
    ``fast_build`` selects an algorithm in the reference and does not change the index."""
    return _bloom_build(feature_ids, feature_offsets, feature_values, b_multiplier, 0, k)


def bloom_index_build_fixed(feature_ids: Tensor, feature_offsets: Tensor, feature_values: Tensor,
                            bits_per_doc: int, k: int, fast_build: bool = False) -> tuple[Tensor, Tensor]:
    """``st::bloom_index_build_fixed``: every bundle ``bits_per_doc`` bits per doc."""
    _check(bits_per_doc > 0, "bits_per_doc must be positive")
    return _bloom_build(feature_ids, feature_offsets, feature_values, 2.0, bits_per_doc, k)


FUSED_PARTIAL_SCHEMA = (
    "fused_kmean_ann_with_partial_masks(Tensor cluster_offsets, Tensor cluster_ids, Tensor cluster_length, "
    "Tensor embeddings, Tensor queries, int max_tensor_size_per_row, Tensor partial_mask_column_counts_cumsum, "
    "Tensor partial_mask_first_item_offset_in_column, Tensor partial_mask_column_results, "
    "int invalid_index_value=-1, int divisor_for_int8=-1, Tensor? filtering_bit_index=None, "
    "Tensor? per_embedding_scale=None, Tensor? cluster_warp_size=None, "
    "Tensor? cluster_warp_rounded_length_cumsum=None, Tensor? cluster_remaining_length_cumsum=None, "
    "Tensor? cluster_warp_size_cumsum=None, int total_cluster_rounded_warps=0, "
    "int total_cluster_remaining_warps=0) -> (Tensor, Tensor)"
)
FUSED_KMEAN_ANN_SCHEMA = (
    "fused_kmean_ann(Tensor cluster_offsets, Tensor cluster_ids, Tensor cluster_length, Tensor embeddings, "
    "Tensor queries, int max_tensor_size_per_row, Tensor? filtering_bit_mask=None, int invalid_index_value=-1, "
    "int divisor_for_int8=-1, Tensor? filtering_bit_index=None, Tensor? per_embedding_scale=None) "
    "-> (Tensor, Tensor)"
)


def fused_kmean_ann(cluster_offsets: Tensor, cluster_ids: Tensor, cluster_length: Tensor, embeddings: Tensor,
                    queries: Tensor, max_tensor_size_per_row: int, filtering_bit_mask: Tensor | None = None,
                    invalid_index_value: int = -1, divisor_for_int8: int = -1,
                    filtering_bit_index: Tensor | None = None,
                    per_embedding_scale: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """``st::fused_kmean_ann`` on int8 codes (the form the reference adapter's official path
    calls, retrieve/src/retrieve/ops/official/adapter.py:289-335): ``(raw [B, W] int32 or
    fp16, idx [B, W] int32)``, ``W = round_up(max_tensor_size_per_row, 32)``, in the CUDA
    scorer's slot order, ``INT32_MIN`` / ``-65504`` and ``invalid_index_value`` where nothing
    was scored. ``filtering_bit_index`` [B] makes row ``b`` read mask row
    ``filtering_bit_index[b]``; ``per_embedding_scale`` (fp16 [N], a per-doc divisor in the
    divisor's place) gives fp16 ``fp16(fp32(fp16(dot)) / fp32(scale))``, the CUDA scorer's order.
    Float embeddings (fp32 / fp16 / bf16, queries of the same dtype) give raw scores of their
    own type by the CUDA scorer's fused multiply-add chains."""
    return _fused(cluster_offsets, cluster_ids, cluster_length, embeddings, queries, max_tensor_size_per_row,
                  filtering_bit_mask, None, invalid_index_value, divisor_for_int8, filtering_bit_index,
                  per_embedding_scale, "st::fused_kmean_ann")


def fused_kmean_ann_with_partial_masks(
        cluster_offsets: Tensor, cluster_ids: Tensor, cluster_length: Tensor, embeddings: Tensor, queries: Tensor,
        max_tensor_size_per_row: int, partial_mask_column_counts_cumsum: Tensor,
        partial_mask_first_item_offset_in_column: Tensor, partial_mask_column_results: Tensor,
        invalid_index_value: int = -1, divisor_for_int8: int = -1, filtering_bit_index: Tensor | None = None,
        per_embedding_scale: Tensor | None = None, cluster_warp_size: Tensor | None = None,
        cluster_warp_rounded_length_cumsum: Tensor | None = None,
        cluster_remaining_length_cumsum: Tensor | None = None, cluster_warp_size_cumsum: Tensor | None = None,
        total_cluster_rounded_warps: int = 0, total_cluster_remaining_warps: int = 0) -> tuple[Tensor, Tensor]:
    """``st::fused_kmean_ann_with_partial_masks`` on int8 codes (fused_kmean_ann_cuda.cu:661-845):
    ``fused_kmean_ann`` with the bloom of the probed clusters only, the triple of
    ``bloom_index_search_batch_return_partial_response`` for the same ``(cluster_offsets[cluster_ids],
    cluster_length)`` ranges: probe ``j`` of row ``b`` keeps its ``i``-th doc when bit
    ``first[b P + j] + i`` of the words from ``cumsum[b P + j - 1]`` on is set (high bit first).
    The slot layout follows from ``cluster_length``; the precomputed warp cumsums of
    ``st::probe_prep`` (``cluster_warp_size`` ... ``total_cluster_remaining_warps``) are accepted and
    not read."""
    partial = (partial_mask_column_counts_cumsum, partial_mask_first_item_offset_in_column,
               partial_mask_column_results)
    return _fused(cluster_offsets, cluster_ids, cluster_length, embeddings, queries, max_tensor_size_per_row, None,
                  partial, invalid_index_value, divisor_for_int8, filtering_bit_index, per_embedding_scale,
                  "st::fused_kmean_ann_with_partial_masks")


FUSED_PARTIAL_MULTIPLE_SCHEMA = (
    "fused_kmean_ann_with_partial_masks_multiple(Tensor queries, Tensor[] list_cluster_offsets, "
    "Tensor[] list_selected_cluster_ids, Tensor[] list_selected_cluster_lengths, Tensor[] list_embeddings, "
    "int[] list_max_tensor_size_per_row, Tensor[] list_partial_mask_column_counts_cumsum, "
    "Tensor[] list_partial_mask_first_item_offset_in_column, Tensor[] list_partial_mask_column_results, "
    "int invalid_index_value=-1, int divisor_for_int8=-1, Tensor? filtering_bit_index=None, "
    "Tensor[]? list_per_embedding_scale=None, bool fuse=False) -> (Tensor[], Tensor[])"
)


def fused_kmean_ann_with_partial_masks_multiple(
        queries: Tensor, list_cluster_offsets: list[Tensor], list_selected_cluster_ids: list[Tensor],
        list_selected_cluster_lengths: list[Tensor], list_embeddings: list[Tensor],
        list_max_tensor_size_per_row: list[int], list_partial_mask_column_counts_cumsum: list[Tensor],
        list_partial_mask_first_item_offset_in_column: list[Tensor], list_partial_mask_column_results: list[Tensor],
        invalid_index_value: int = -1, divisor_for_int8: int = -1, filtering_bit_index: Tensor | None = None,
        list_per_embedding_scale: list[Tensor] | None = None,
        fuse: bool = False) -> tuple[list[Tensor], list[Tensor]]:
    """``st::fused_kmean_ann_with_partial_masks_multiple`` (fused_kmean_ann.cpp:438-456; CUDA
    fused_kmean_ann_cuda.cu:2503-2600): the partial-mask scorer over an index held in chunks, one
    ``(raw, idx)`` pair per chunk, each the single op's result on that chunk. ``fuse`` groups the
    reference's launches and does not change the results; here every chunk is one call."""
    n = len(list_cluster_offsets)
    for name, lst in (("list_selected_cluster_ids", list_selected_cluster_ids),
                      ("list_selected_cluster_lengths", list_selected_cluster_lengths),
                      ("list_embeddings", list_embeddings),
                      ("list_max_tensor_size_per_row", list_max_tensor_size_per_row),
                      ("list_partial_mask_column_counts_cumsum", list_partial_mask_column_counts_cumsum),
                      ("list_partial_mask_first_item_offset_in_column", list_partial_mask_first_item_offset_in_column),
                      ("list_partial_mask_column_results", list_partial_mask_column_results)):
        _check(len(lst) == n, f"{name} must have the same size as list_cluster_offsets")
    if list_per_embedding_scale is not None:
        _check(len(list_per_embedding_scale) == n, "list_per_embedding_scale must have the same size as "
                                                   "list_cluster_offsets")
    raws, idxs = [], []
    for i in range(n):
        raw, idx = fused_kmean_ann_with_partial_masks(
            list_cluster_offsets[i], list_selected_cluster_ids[i], list_selected_cluster_lengths[i],
            list_embeddings[i], queries, int(list_max_tensor_size_per_row[i]),
            list_partial_mask_column_counts_cumsum[i], list_partial_mask_first_item_offset_in_column[i],
            list_partial_mask_column_results[i], invalid_index_value, divisor_for_int8, filtering_bit_index,
            None if list_per_embedding_scale is None else list_per_embedding_scale[i])
        raws.append(raw)
        idxs.append(idx)
    return raws, idxs


def _fused(cluster_offsets, cluster_ids, cluster_length, embeddings, queries, max_tensor_size_per_row,
           filtering_bit_mask, partial, invalid_index_value, divisor_for_int8, filtering_bit_index,
           per_embedding_scale, what):
    codes = {torch.int8: _lib.RB_I8, torch.float32: _lib.RB_F32, torch.float16: _lib.RB_F16,
             torch.bfloat16: _lib.RB_BF16}
    _check(embeddings.dtype in codes, f"{what}: unsupported scalar type {embeddings.dtype}")
    _check(queries.dtype == embeddings.dtype, f"{what}: queries must have the embeddings' dtype")
    is_int8 = embeddings.dtype == torch.int8
    for name, t in (("cluster_offsets", cluster_offsets), ("cluster_ids", cluster_ids),
                    ("cluster_length", cluster_length), ("embeddings", embeddings), ("queries", queries)):
        _check(t.is_cuda and t.is_contiguous(), f"{name} must be a contiguous CUDA tensor")
    _check(cluster_offsets.dim() == 1 and cluster_ids.dim() == 2 and cluster_length.dim() == 2
           and embeddings.dim() == 2 and queries.dim() == 2, "bad ranks")
    _check(cluster_ids.shape == cluster_length.shape and cluster_ids.shape[0] == queries.shape[0]
           and embeddings.shape[1] == queries.shape[1], "shape mismatch")
    dev = queries.device
    b, d = queries.shape
    p = cluster_ids.shape[1]
    width = (int(max_tensor_size_per_row) + 31) // 32 * 32
    offs = cluster_offsets.to(torch.int64).contiguous()
    cids = cluster_ids.to(torch.int64).contiguous()
    clen = cluster_length.to(torch.int64).contiguous()
    scale = None
    if per_embedding_scale is not None:  # the reference's checks, fused_kmean_ann_cuda.cu:2186-2200
        _check(per_embedding_scale.is_cuda, "per_embedding_scale is not on GPU")
        _check(per_embedding_scale.is_contiguous(), "per_embedding_scale is not contiguous")
        _check(per_embedding_scale.dim() == 1, "per_embedding_scale is not 1D")
        _check(per_embedding_scale.shape[0] == embeddings.shape[0],
               "per_embedding_scale size does not match embedding size")
        _check(per_embedding_scale.dtype == torch.float16, "per_embedding_scale is not half")
        scale = per_embedding_scale
    rows_index = None
    if filtering_bit_index is not None:  # row b reads mask row filtering_bit_index[b]
        _check(filtering_bit_index.is_cuda and filtering_bit_index.dim() == 1 and filtering_bit_index.shape[0] == b,
               "filtering_bit_index must be a 1-D CUDA tensor of one mask row per query row")
        rows_index = filtering_bit_index.to(torch.int64).contiguous()
    half = divisor_for_int8 != -1 or scale is not None
    raw_dtype = (torch.float16 if half else torch.int32) if is_int8 else embeddings.dtype
    raw = torch.empty((b, width), dtype=raw_dtype, device=dev)
    idx = torch.empty((b, width), dtype=torch.int32, device=dev)
    mask = None
    if filtering_bit_mask is not None:
        _check(filtering_bit_mask.dim() == 2 and (rows_index is not None or filtering_bit_mask.shape[0] == b),
               "filtering_bit_mask must be [B, W] (or [R, W] with filtering_bit_index)")
        mask = filtering_bit_mask.to(device=dev, dtype=torch.int64).contiguous()
    mask_rows = 0 if mask is None else mask.shape[0]
    if partial is not None:
        cumsum, first, words = partial
        for name, t in (("partial_mask_column_counts_cumsum", cumsum),
                        ("partial_mask_first_item_offset_in_column", first),
                        ("partial_mask_column_results", words)):
            _check(t.is_cuda, f"{name} must be a CUDA tensor")
        ranges = cumsum.numel()
        _check(first.numel() == ranges and (ranges == b * p or (rows_index is not None and p > 0 and ranges % p == 0)),
               "the partial mask needs one column cumsum and one bit offset per (row, probe) "
               "(per (mask row, probe) with filtering_bit_index)")
        mask_rows = ranges // p if p else b
        cumsum = cumsum.to(torch.int32).contiguous()
        first = first.to(torch.int8).contiguous()
        words = words.to(torch.int64).contiguous()
    if b == 0 or width == 0:
        return raw, idx
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _call(lib.rb_st_fused_kmean_ann_workspace_size(b, p, int(max_tensor_size_per_row), ctypes.byref(nbytes)), what)
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
    common = (_ptr(offs), offs.numel() - 1 if offs.numel() else 0, _ptr(cids), _ptr(clen), p, _ptr(embeddings),
              embeddings.shape[0], _ptr(queries), codes[embeddings.dtype], b, d, int(max_tensor_size_per_row))
    tail = (_ptr(scale), int(invalid_index_value), int(divisor_for_int8), _ptr(raw), _ptr(idx), _ptr(ws), ws.numel(),
            _stream(dev))
    if partial is None:
        rc = lib.rb_st_fused_kmean_ann(*common, _ptr(mask), mask_rows, 0 if mask is None else mask.shape[1],
                                       _ptr(rows_index), *tail)
    else:
        rc = lib.rb_st_fused_kmean_ann_with_partial_masks(*common, _ptr(cumsum), _ptr(first), _ptr(words),
                                                          words.numel(), mask_rows, _ptr(rows_index), *tail)
    _call(rc, what)
    return raw, idx


def _fake_fused_kmean_ann(cluster_offsets, cluster_ids, cluster_length, embeddings, queries, max_tensor_size_per_row,
                          filtering_bit_mask=None, invalid_index_value=-1, divisor_for_int8=-1,
                          filtering_bit_index=None, per_embedding_scale=None):
    width = (int(max_tensor_size_per_row) + 31) // 32 * 32
    b = queries.shape[0]
    dt = torch.int32 if divisor_for_int8 == -1 and per_embedding_scale is None else torch.float16
    if embeddings.dtype != torch.int8:
        dt = embeddings.dtype
    return queries.new_empty((b, width), dtype=dt), queries.new_empty((b, width), dtype=torch.int32)


def _fake_fused_partial(cluster_offsets, cluster_ids, cluster_length, embeddings, queries, max_tensor_size_per_row,
                        *args, invalid_index_value=-1, divisor_for_int8=-1, **kwargs):
    # positional form: args = (cumsum, first, words, invalid_index_value, divisor_for_int8,
    # filtering_bit_index, per_embedding_scale, ...)
    if len(args) >= 5:
        divisor_for_int8 = args[4]
    scale = args[6] if len(args) >= 7 else kwargs.get("per_embedding_scale")
    return _fake_fused_kmean_ann(cluster_offsets, cluster_ids, cluster_length, embeddings, queries,
                                 max_tensor_size_per_row, divisor_for_int8=divisor_for_int8, per_embedding_scale=scale)


def _fake_fused_partial_multiple(queries, list_cluster_offsets, list_selected_cluster_ids,
                                 list_selected_cluster_lengths, list_embeddings, list_max_tensor_size_per_row,
                                 *args, invalid_index_value=-1, divisor_for_int8=-1, **kwargs):
    if len(args) >= 5:
        divisor_for_int8 = args[4]
    scales = args[6] if len(args) >= 7 else kwargs.get("list_per_embedding_scale")
    b = queries.shape[0]
    dt = torch.int32 if divisor_for_int8 == -1 and scales is None else torch.float16
    if list_embeddings and list_embeddings[0].dtype != torch.int8:
        dt = list_embeddings[0].dtype
    widths = [(int(m) + 31) // 32 * 32 for m in list_max_tensor_size_per_row]
    return ([queries.new_empty((b, w), dtype=dt) for w in widths],
            [queries.new_empty((b, w), dtype=torch.int32) for w in widths])


def _fake_bloom(feature_ids, feature_offsets, feature_values, *args, **kwargs):
    # the index length depends on the data (the reference's builders read it back too)
    n = (feature_offsets.shape[0] - 1) // max(feature_ids.shape[0], 1)
    ctx = torch.library.get_ctx()
    words = ctx.new_dynamic_size()
    return (feature_values.new_empty((words,), dtype=torch.int64),
            feature_values.new_empty(((n + 2047) // 2048 + 1,), dtype=torch.int64))


def _fake_search(query, probe_ids, cluster_offsets, cluster_sizes, item_codes, sort_perm, global_scale, k,
                 max_tensor_size_per_row, *args, **kwargs):
    b = query.shape[0]
    return query.new_empty((b, k), dtype=torch.int64), query.new_empty((b, k), dtype=torch.float32)


def _fake_probe_prep(query, probe_ids, cluster_offsets, cluster_sizes):
    rows, n_probe = probe_ids.shape
    i64 = probe_ids.new_empty((rows, n_probe), dtype=torch.int64)
    return (
        query.new_empty(query.shape, dtype=torch.int8),
        query.new_empty((rows,), dtype=torch.float32),
        i64,
        torch.empty_like(i64),
        torch.empty_like(i64),
        probe_ids.new_empty((rows * n_probe,), dtype=torch.int32),
        probe_ids.new_empty((rows, n_probe), dtype=torch.int32),
        probe_ids.new_empty((rows * n_probe,), dtype=torch.int32),
        probe_ids.new_empty((rows * n_probe,), dtype=torch.int32),
    )


_lib.lib()  # no fallback: a missing library fails the import
_LIBRARY = torch.library.Library("st", "FRAGMENT")


def _defined(name: str) -> bool:
    """Whether a loaded library (the reference's CPU build, say) already defines ``st::<name>``."""
    return hasattr(torch.ops.st, name)


def _register() -> None:
    for name, schema, impl, fake in (("search", SEARCH_SCHEMA, search, _fake_search),
                                     ("probe_prep", PROBE_PREP_SCHEMA, probe_prep, _fake_probe_prep),
                                     ("bloom_index_build", BLOOM_BUILD_SCHEMA, bloom_index_build, _fake_bloom),
                                     ("bloom_index_build_fixed", BLOOM_BUILD_FIXED_SCHEMA, bloom_index_build_fixed,
                                      _fake_bloom),
                                     ("fused_kmean_ann", FUSED_KMEAN_ANN_SCHEMA, fused_kmean_ann,
                                      _fake_fused_kmean_ann),
                                     ("fused_kmean_ann_with_partial_masks", FUSED_PARTIAL_SCHEMA,
                                      fused_kmean_ann_with_partial_masks, _fake_fused_partial),
                                     ("fused_kmean_ann_with_partial_masks_multiple", FUSED_PARTIAL_MULTIPLE_SCHEMA,
                                      fused_kmean_ann_with_partial_masks_multiple, _fake_fused_partial_multiple),
                                     *st_bloom.OPS, *st_select.OPS):
        ours = not _defined(name)
        if ours:
            _LIBRARY.define(schema)
        _LIBRARY.impl(name, impl, "CUDA")
        if ours:
            torch.library.register_fake(f"st::{name}", fake, lib=_LIBRARY)
    # the host parser: for CPU ks tensors too, unless a loaded build (the reference's CPU
    # ops) already serves the CPU key with the same parser
    name = "parse_expression_query_batch"
    ours = not _defined(name)
    if ours:
        _LIBRARY.define(st_bloom.PARSE_SCHEMA)
        _LIBRARY.impl(name, st_bloom.parse_expression_query_batch, "CPU")
    _LIBRARY.impl(name, st_bloom.parse_expression_query_batch, "CUDA")


_register()
