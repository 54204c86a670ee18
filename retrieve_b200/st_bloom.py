"""SilverTorch's bloom index searches as ``torch.ops.st`` CUDA ops on ``libretrieve_b200.so``.

The upstream-shaped searches of the reference's loader list
(retrieve/src/retrieve/ops/official/__init__.py:46-54), schemas as the reference pins them
(retrieve/tests/parity/test_official.py:65-102; silvertorch/ops/csrc/bloom_index_search.cpp
:543-601):

* ``bloom_index_search_batch`` / ``_prepared``: every plan over every 64-doc column of the
  bundle-major index, the packed int64 ``[Q, n_bundles * 32]`` words (doc ``64 c + i`` at bit
  ``63 - i``) or bool ``[Q, n_bundles * 2048]``;
* ``generate_column_info_for_clusters``: per probed range ``(start, length)`` its column count,
  first column and bit offset;
* ``bloom_index_search_batch_return_partial_response`` / ``_prepared``: the words of only the
  probed clusters' columns, with the inclusive column cumsum and the bit offsets, the triple
  ``fused_kmean_ann_with_partial_masks`` reads.

Plans come as the parser's ``(data int8, offsets int64)`` (read on the host, as the reference's
CUDA ops decode them, bloom_index_search_cuda.cu:1614-1617) or prepared on the device (the blob
of ``adapter.prepare_plans``: per plan slot 8 offsets, then the data). Limits: ``1 <= k <= 10``
and plan stacks at most 16 deep. Errors raise ``RuntimeError``.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch
from torch import Tensor

from retrieve_b200 import _lib
from retrieve_b200._st_common import _call, _check, _ptr, _stream

BLOOM_SEARCH_SCHEMA = (
    "bloom_index_search_batch(Tensor bloom_index, Tensor bloom_bundle_b_offsets, "
    "Tensor bloom_query_plans_data, Tensor bloom_query_plans_offsets, int k, int hash_k, "
    "bool return_bool_mask=True) -> Tensor"
)
BLOOM_SEARCH_PREPARED_SCHEMA = (
    "bloom_index_search_batch_prepared(Tensor bloom_index, Tensor bloom_bundle_b_offsets, Tensor plans, "
    "int plan_count, int max_stack_size, int k, int hash_k, bool return_bool_mask=False) -> Tensor"
)
COLUMN_INFO_SCHEMA = (
    "generate_column_info_for_clusters(Tensor selected_cluster_offsets, Tensor selected_cluster_lengths) "
    "-> (Tensor, Tensor, Tensor)"
)
PARTIAL_SCHEMA = (
    "bloom_index_search_batch_return_partial_response(Tensor bloom_index, Tensor bloom_bundle_b_offsets, "
    "Tensor bloom_query_plans_data, Tensor bloom_query_plans_offsets, Tensor selected_cluster_offsets, "
    "Tensor selected_cluster_lengths, int k, int hash_k, Tensor? query_plan_index=None) "
    "-> (Tensor, Tensor, Tensor)"
)
PARTIAL_PREPARED_SCHEMA = (
    "bloom_index_search_batch_return_partial_response_prepared(Tensor bloom_index, "
    "Tensor bloom_bundle_b_offsets, Tensor plans, int plan_count, int max_stack_size, "
    "Tensor selected_cluster_offsets, Tensor selected_cluster_lengths, int k, int hash_k, "
    "Tensor? query_plan_index, int max_columns) -> (Tensor, Tensor, Tensor)"
)

PARTIAL_MULTIPLE_SCHEMA = (
    "bloom_index_search_batch_return_partial_response_multiple(Tensor[] list_bloom_index, "
    "Tensor[] list_bloom_bundle_b_offsets, Tensor bloom_query_plans_data, Tensor bloom_query_plans_offsets, "
    "Tensor[] list_selected_cluster_offsets, Tensor[] list_selected_cluster_lengths, int k, int hash_k, "
    "Tensor? query_plan_index=None, bool fuse=False) -> (Tensor[], Tensor[], Tensor[])"
)
PARSE_SCHEMA = (
    "parse_expression_query_batch(str[] expressions, Tensor silvertorch_ks, int bloom_hash_k, "
    "bool return_query_plan=True, int max_sub_queries=5) -> (int, Tensor[])"
)

DOCS_PER_BUNDLE = 2048
COLUMNS_PER_BUNDLE = 32
_OP_AND, _OP_OR, _OP_NOT, _OP_TERM, _OP_EMPTY = 1, 2, 3, 4, 5


def plan_stack_depth(raw: np.ndarray, offs: np.ndarray) -> int:
    """The deepest operand stack any plan reaches when evaluated in postfix order: a term or
    ``EMPTY`` pushes one word, ``AND`` / ``OR`` pop as many children as their operator-offset
    range holds and push one, ``NOT`` replaces the top. ``raw`` is the parser's data bytes,
    ``offs`` its eight byte offsets a plan (bloom_index_util.cpp:82-125)."""
    depth = 0
    for p in range(offs.size // 8):
        o = offs[8 * p : 8 * p + 8]
        if (o < 0).any() or (o[1::2] > raw.size).any() or (o[0::2] > o[1::2]).any() or o[2] % 4:
            continue  # a malformed plan matches nothing on the device; it needs no stack
        ops = raw[o[0] : o[1]]
        op_off = raw[o[2] : o[3] - (o[3] - o[2]) % 4].view(np.int32)
        sp = 0
        for j, op in enumerate(ops.tolist()):
            if op in (_OP_TERM, _OP_EMPTY):
                sp += 1
            elif op in (_OP_AND, _OP_OR):
                children = int(op_off[j + 1]) - int(op_off[j]) if j + 1 < op_off.size else 0
                sp = max(sp - max(children, 0), 0) + 1
            depth = max(depth, sp)
    return depth


def prepare_plans(data: Tensor, offsets: Tensor, device: torch.device) -> tuple[Tensor, int, int]:
    """The parser's ``(data, offsets)`` as the device blob the searches read:
    ``(blob int64 [8 Q + ceil(bytes / 8)], Q, max stack depth)``."""
    raw = np.ascontiguousarray(data.detach().cpu().contiguous().view(torch.uint8).numpy().reshape(-1))
    offs = np.ascontiguousarray(offsets.detach().cpu().to(torch.int64).numpy().reshape(-1))
    _check(offs.size % 8 == 0, "bloom_query_plans_offsets must hold 8 offsets a plan")
    slots = offs.size // 8
    blob = np.zeros(8 * slots + (raw.size + 7) // 8, dtype=np.int64)
    blob[: offs.size] = offs
    blob[8 * slots :].view(np.uint8)[: raw.size] = raw
    return torch.from_numpy(blob).to(device), slots, plan_stack_depth(raw, offs)


def parse_expression_query_batch(expressions: list[str], silvertorch_ks: Tensor, bloom_hash_k: int,
                                 return_query_plan: bool = True,
                                 max_sub_queries: int = 5) -> tuple[int, list[Tensor]]:
    """``st::parse_expression_query_batch`` (expression_query_parser.cpp:395-430) by the
    library's host parser: ``(max_stack_size, [plans_data int8, plans_offsets int64])`` on the
    CPU, byte-identical to the reference's; both tensors empty when ``return_query_plan`` is
    false. ``silvertorch_ks`` is accepted and ignored, as upstream. A malformed expression
    raises ``RuntimeError``."""
    raw = [e.encode("utf-8") for e in expressions]
    n = len(raw)
    bufs = (ctypes.c_char_p * max(n, 1))(*raw) if n else None
    lengths = (ctypes.c_int64 * max(n, 1))(*[len(r) for r in raw])
    nbytes, stack = ctypes.c_int64(0), ctypes.c_int64(0)
    lib = _lib.lib()
    what = "st::parse_expression_query_batch"
    _call(lib.rb_st_parse_expression_batch(bufs, lengths, n, int(bloom_hash_k), int(max_sub_queries), None, 0, None,
                                           ctypes.byref(nbytes), ctypes.byref(stack)), what)
    if not return_query_plan:
        return int(stack.value), [torch.empty(0, dtype=torch.int8), torch.empty(0, dtype=torch.int64)]
    data = torch.empty(int(nbytes.value), dtype=torch.int8)
    offsets = torch.empty(8 * n, dtype=torch.int64)
    _call(lib.rb_st_parse_expression_batch(bufs, lengths, n, int(bloom_hash_k), int(max_sub_queries), _ptr(data),
                                           data.numel(), _ptr(offsets), ctypes.byref(nbytes), ctypes.byref(stack)),
          what)
    return int(stack.value), [data, offsets]


def _index_args(bloom_index: Tensor, bloom_bundle_b_offsets: Tensor):
    _check(bloom_index.is_cuda, "bloom_index must be a CUDA tensor")
    _check(bloom_index.dim() == 1, "bloom_index must be 1-D")
    _check(bloom_index.is_contiguous(), "bloom_index must be contiguous")
    _check(bloom_index.dtype == torch.int64, "bloom_index must be int64")
    boff = bloom_bundle_b_offsets.to(device=bloom_index.device, dtype=torch.int64).contiguous()
    _check(boff.dim() == 1 and boff.numel() >= 1, "bloom_bundle_b_offsets must be 1-D [n_bundles + 1]")
    return boff, boff.numel() - 1


def _search(bloom_index, boff, n_bundles, blob, slots, max_stack, k, hash_k, return_bool_mask, what):
    dev = bloom_index.device
    n_cols = n_bundles * COLUMNS_PER_BUNDLE
    if return_bool_mask:
        out = torch.empty((slots, n_cols * 64), dtype=torch.bool, device=dev)
    else:
        out = torch.empty((slots, n_cols), dtype=torch.int64, device=dev)
    _call(_lib.lib().rb_st_bloom_search(
        _ptr(bloom_index), bloom_index.numel(), _ptr(boff), n_bundles, _ptr(blob), blob.numel(), slots,
        int(max_stack), int(k), int(hash_k), int(bool(return_bool_mask)), _ptr(out), _stream(dev)), what)
    return out


def bloom_index_search_batch(bloom_index: Tensor, bloom_bundle_b_offsets: Tensor, bloom_query_plans_data: Tensor,
                             bloom_query_plans_offsets: Tensor, k: int, hash_k: int,
                             return_bool_mask: bool = True) -> Tensor:
    """``st::bloom_index_search_batch`` on the device (bloom_index_search_cuda.cu:1598-1640)."""
    boff, n_bundles = _index_args(bloom_index, bloom_bundle_b_offsets)
    blob, slots, depth = prepare_plans(bloom_query_plans_data, bloom_query_plans_offsets, bloom_index.device)
    return _search(bloom_index, boff, n_bundles, blob, slots, depth, k, hash_k, return_bool_mask,
                   "st::bloom_index_search_batch")


def bloom_index_search_batch_prepared(bloom_index: Tensor, bloom_bundle_b_offsets: Tensor, plans: Tensor,
                                      plan_count: int, max_stack_size: int, k: int, hash_k: int,
                                      return_bool_mask: bool = False) -> Tensor:
    """``st::bloom_index_search_batch_prepared`` (bloom_index_search_cuda.cu:1832-1859): plans
    already on the device, no host work."""
    boff, n_bundles = _index_args(bloom_index, bloom_bundle_b_offsets)
    _check(plans.is_cuda and plans.dtype == torch.int64, "plans must be a CUDA int64 tensor")
    blob = plans.contiguous()
    return _search(bloom_index, boff, n_bundles, blob, int(plan_count), max_stack_size, k, hash_k,
                   return_bool_mask, "st::bloom_index_search_batch_prepared")


def _ranges(selected_cluster_offsets: Tensor, selected_cluster_lengths: Tensor, two_d: bool):
    for name, t in (("selected_cluster_offsets", selected_cluster_offsets),
                    ("selected_cluster_lengths", selected_cluster_lengths)):
        _check(t.is_cuda, f"{name} must be a CUDA tensor")
        _check(t.dtype == torch.int64, f"{name} dtype must be Long")
        if two_d:
            _check(t.dim() == 2, f"{name} dim must be 2, but got {t.dim()}")
    _check(selected_cluster_offsets.shape == selected_cluster_lengths.shape,
           "selected_cluster_offsets must have same shape with selected_cluster_lengths")
    return selected_cluster_offsets.contiguous(), selected_cluster_lengths.contiguous()


def _column_info(offs: Tensor, lens: Tensor, with_cumsum: bool):
    n = offs.numel()
    dev = offs.device
    counts = torch.empty(n, dtype=torch.int32, device=dev)
    starts = torch.empty(n, dtype=torch.int32, device=dev)
    first = torch.empty(n, dtype=torch.int8, device=dev)
    cumsum = torch.empty(n, dtype=torch.int32, device=dev) if with_cumsum else None
    _call(_lib.lib().rb_st_bloom_column_info(_ptr(offs), _ptr(lens), n, _ptr(counts), _ptr(starts), _ptr(first),
                                             _ptr(cumsum), _stream(dev)), "st::generate_column_info_for_clusters")
    return counts, starts, first, cumsum


def generate_column_info_for_clusters(selected_cluster_offsets: Tensor,
                                      selected_cluster_lengths: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """``st::generate_column_info_for_clusters`` on the device: ``(column_counts int32,
    start_column_ids int32, first_item_offsets_in_column int8)``, one entry per range."""
    offs, lens = _ranges(selected_cluster_offsets, selected_cluster_lengths, two_d=False)
    _check(offs.dim() in (1, 2), f"selected_cluster_offsets must be 1D or 2D, got {offs.dim()}D")
    counts, starts, first, _ = _column_info(offs, lens, with_cumsum=False)
    return counts, starts, first


def _partial(bloom_index, bloom_bundle_b_offsets, blob, slots, max_stack, selected_cluster_offsets,
             selected_cluster_lengths, k, hash_k, query_plan_index, max_columns, what):
    # max_columns None: the parser's plans, one a row unless query_plan_index maps rows to plans
    # (bloom_index_search.cpp:300-307); else prepared plan slots, row b reading slot b
    boff, n_bundles = _index_args(bloom_index, bloom_bundle_b_offsets)
    offs, lens = _ranges(selected_cluster_offsets, selected_cluster_lengths, two_d=True)
    b, p = lens.shape
    dev = bloom_index.device
    qpi = None
    if query_plan_index is not None:
        _check(query_plan_index.is_cuda, "query_plan_index must be a CUDA tensor")
        _check(query_plan_index.dim() == 1, f"query_plan_index dim must be 1, but got {query_plan_index.dim()}")
        _check(query_plan_index.shape[0] == b, "query_plan count must be same with selected_cluster size[0]")
        qpi = query_plan_index.to(torch.int64).contiguous()
    elif max_columns is None:
        _check(slots == b, f"query_plan_count must be equal to query_count if no query_plan_index, "
                           f"but got {slots} vs {b}")
    _, starts, first, cumsum = _column_info(offs, lens, with_cumsum=True)
    if max_columns is None:  # the reference's unprepared form sizes the words from the total
        max_columns = int(cumsum[-1].item()) if cumsum.numel() else 0
    words = torch.empty(int(max_columns), dtype=torch.int64, device=dev)
    _call(_lib.lib().rb_st_bloom_partial_search(
        _ptr(bloom_index), bloom_index.numel(), _ptr(boff), n_bundles, _ptr(blob), blob.numel(), slots,
        int(max_stack), _ptr(qpi), b, p, _ptr(cumsum), _ptr(starts), int(k), int(hash_k), _ptr(words),
        words.numel(), _stream(dev)), what)
    return cumsum, first, words


def bloom_index_search_batch_return_partial_response(
        bloom_index: Tensor, bloom_bundle_b_offsets: Tensor, bloom_query_plans_data: Tensor,
        bloom_query_plans_offsets: Tensor, selected_cluster_offsets: Tensor, selected_cluster_lengths: Tensor,
        k: int, hash_k: int, query_plan_index: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """``st::bloom_index_search_batch_return_partial_response`` on the device
    (bloom_index_search_cuda.cu:1780-1830): ``(column_counts_cumsum int32 [B P],
    first_item_offset_in_column int8 [B P], column_mask_response int64 [total columns])``; the
    total is read back once to size the words, as the reference's op does."""
    blob, slots, depth = prepare_plans(bloom_query_plans_data, bloom_query_plans_offsets, bloom_index.device)
    return _partial(bloom_index, bloom_bundle_b_offsets, blob, slots, depth, selected_cluster_offsets,
                    selected_cluster_lengths, k, hash_k, query_plan_index, None,
                    "st::bloom_index_search_batch_return_partial_response")


def bloom_index_search_batch_return_partial_response_prepared(
        bloom_index: Tensor, bloom_bundle_b_offsets: Tensor, plans: Tensor, plan_count: int, max_stack_size: int,
        selected_cluster_offsets: Tensor, selected_cluster_lengths: Tensor, k: int, hash_k: int,
        query_plan_index: Tensor | None, max_columns: int) -> tuple[Tensor, Tensor, Tensor]:
    """The prepared form (bloom_index_search_cuda.cu:1861-1944): no host sync, the words a
    static ``max_columns`` long with a zero tail."""
    _check(plans.is_cuda and plans.dtype == torch.int64, "plans must be a CUDA int64 tensor")
    _check(int(max_columns) >= 0, "max_columns must be >= 0")
    return _partial(bloom_index, bloom_bundle_b_offsets, plans.contiguous(), int(plan_count), max_stack_size,
                    selected_cluster_offsets, selected_cluster_lengths, k, hash_k, query_plan_index,
                    int(max_columns), "st::bloom_index_search_batch_return_partial_response_prepared")


def bloom_index_search_batch_return_partial_response_multiple(
        list_bloom_index: list[Tensor], list_bloom_bundle_b_offsets: list[Tensor], bloom_query_plans_data: Tensor,
        bloom_query_plans_offsets: Tensor, list_selected_cluster_offsets: list[Tensor],
        list_selected_cluster_lengths: list[Tensor], k: int, hash_k: int, query_plan_index: Tensor | None = None,
        fuse: bool = False) -> tuple[list[Tensor], list[Tensor], list[Tensor]]:
    """``st::bloom_index_search_batch_return_partial_response_multiple`` (bloom_index_search.cpp
    :411-474; CUDA bloom_index_search_cuda.cu:2312-2450): the partial search over an index held in
    chunks, the plans read once, one triple per chunk equal to the single op's on that chunk.
    ``fuse`` groups the reference's launches and does not change the results."""
    n = len(list_bloom_index)
    what = "st::bloom_index_search_batch_return_partial_response_multiple"
    _check(n > 0, "bloom_index_search_batch_return_partial_response_multiple: list_bloom_index should not be empty.")
    for name, lst in (("list_bloom_bundle_b_offsets", list_bloom_bundle_b_offsets),
                      ("list_selected_cluster_offsets", list_selected_cluster_offsets),
                      ("list_selected_cluster_lengths", list_selected_cluster_lengths)):
        _check(len(lst) == n, f"list_bloom_index and {name} should have the same size, got {n} vs {len(lst)}")
    _check(list_bloom_index[0].is_cuda, "bloom_index must be a CUDA tensor")
    blob, slots, depth = prepare_plans(bloom_query_plans_data, bloom_query_plans_offsets, list_bloom_index[0].device)
    out = ([], [], [])
    for i in range(n):
        triple = _partial(list_bloom_index[i], list_bloom_bundle_b_offsets[i], blob, slots, depth,
                          list_selected_cluster_offsets[i], list_selected_cluster_lengths[i], k, hash_k,
                          query_plan_index, None, what)
        for acc, t in zip(out, triple):
            acc.append(t)
    return out


# --- fakes (shapes for tracing) ------------------------------------------------------------


def _fake_search(bloom_index, bloom_bundle_b_offsets, data, offsets, k, hash_k, return_bool_mask=True):
    cols = (bloom_bundle_b_offsets.shape[0] - 1) * COLUMNS_PER_BUNDLE
    q = offsets.shape[0] // 8
    if return_bool_mask:
        return bloom_index.new_empty((q, cols * 64), dtype=torch.bool)
    return bloom_index.new_empty((q, cols), dtype=torch.int64)


def _fake_search_prepared(bloom_index, bloom_bundle_b_offsets, plans, plan_count, max_stack_size, k, hash_k,
                          return_bool_mask=False):
    cols = (bloom_bundle_b_offsets.shape[0] - 1) * COLUMNS_PER_BUNDLE
    if return_bool_mask:
        return bloom_index.new_empty((plan_count, cols * 64), dtype=torch.bool)
    return bloom_index.new_empty((plan_count, cols), dtype=torch.int64)


def _fake_column_info(selected_cluster_offsets, selected_cluster_lengths):
    n = selected_cluster_lengths.numel()
    return (selected_cluster_lengths.new_empty((n,), dtype=torch.int32),
            selected_cluster_lengths.new_empty((n,), dtype=torch.int32),
            selected_cluster_lengths.new_empty((n,), dtype=torch.int8))


def _fake_partial(bloom_index, bloom_bundle_b_offsets, data, offsets, selected_cluster_offsets,
                  selected_cluster_lengths, k, hash_k, query_plan_index=None):
    n = selected_cluster_lengths.numel()
    words = torch.library.get_ctx().new_dynamic_size()
    return (selected_cluster_lengths.new_empty((n,), dtype=torch.int32),
            selected_cluster_lengths.new_empty((n,), dtype=torch.int8),
            bloom_index.new_empty((words,), dtype=torch.int64))


def _fake_partial_prepared(bloom_index, bloom_bundle_b_offsets, plans, plan_count, max_stack_size,
                           selected_cluster_offsets, selected_cluster_lengths, k, hash_k, query_plan_index,
                           max_columns):
    n = selected_cluster_lengths.numel()
    return (selected_cluster_lengths.new_empty((n,), dtype=torch.int32),
            selected_cluster_lengths.new_empty((n,), dtype=torch.int8),
            bloom_index.new_empty((max_columns,), dtype=torch.int64))


def _fake_partial_multiple(list_bloom_index, list_bloom_bundle_b_offsets, data, offsets,
                           list_selected_cluster_offsets, list_selected_cluster_lengths, k, hash_k,
                           query_plan_index=None, fuse=False):
    ctx = torch.library.get_ctx()
    outs = ([], [], [])
    for index, lens in zip(list_bloom_index, list_selected_cluster_lengths):
        n = lens.numel()
        outs[0].append(lens.new_empty((n,), dtype=torch.int32))
        outs[1].append(lens.new_empty((n,), dtype=torch.int8))
        outs[2].append(index.new_empty((ctx.new_dynamic_size(),), dtype=torch.int64))
    return outs


OPS = (
    ("bloom_index_search_batch", BLOOM_SEARCH_SCHEMA, bloom_index_search_batch, _fake_search),
    ("bloom_index_search_batch_prepared", BLOOM_SEARCH_PREPARED_SCHEMA, bloom_index_search_batch_prepared,
     _fake_search_prepared),
    ("generate_column_info_for_clusters", COLUMN_INFO_SCHEMA, generate_column_info_for_clusters, _fake_column_info),
    ("bloom_index_search_batch_return_partial_response", PARTIAL_SCHEMA,
     bloom_index_search_batch_return_partial_response, _fake_partial),
    ("bloom_index_search_batch_return_partial_response_prepared", PARTIAL_PREPARED_SCHEMA,
     bloom_index_search_batch_return_partial_response_prepared, _fake_partial_prepared),
    ("bloom_index_search_batch_return_partial_response_multiple", PARTIAL_MULTIPLE_SCHEMA,
     bloom_index_search_batch_return_partial_response_multiple, _fake_partial_multiple),
)
