"""SilverTorch's IVF probe + int8 scoring path, ``st::search``, restated on the
CPU. Test infrastructure: only the tests, ``smoke()`` and the bench's CPU legs
use it, as the checker.

The op (schema silvertorch/ops/csrc/fork_search.cpp:13-41, body
fork_search_cuda.cu:1256-1524), for each query row ``b``:

1. Query prep (fork_search_cuda.cu:680-700): the row quantized to int8 exactly
   as ``quantize_int8`` evaluates on a CUDA tensor (``oracle.knn.quantize_int8``:
   the code quotient in fp64 rounded to fp32; the scale
   ``abs_max * fp32(1/127)``).
2. Candidates: the sorted-table positions of the probed clusters
   ``probe_ids[b, :]`` (cluster ``c`` holds positions
   ``cluster_offsets[c] .. cluster_offsets[c] + cluster_sizes[c]``). The scorer
   writes them into a row of ``width = round_up(max_tensor_size_per_row, 32)``
   slots in its own order: first every probed cluster's warp-aligned prefix
   (``32 * (len // 32)`` positions), cluster by cluster in probe order, then
   every cluster's remainder (``len % 32`` positions), in probe order
   (silvertorch/ops/csrc/fused_kmean_ann_cuda.cu:100-110 and 183-215; the
   prep's cumsums, fork_search_cuda.cu:705-760). ``probe_slots`` gives that
   order; it decides which of several tied candidates is kept.
3. Score per slot: the exact int32 dot of the int8 codes
   (fused_kmean_ann.cpp:60-70); with ``divisor_for_int8 != -1`` the fp16 value
   ``fp16(fp32(dot) / fp32(divisor))`` (fused_kmean_ann.cpp:196-200,
   fused_kmean_ann_cuda.cu:1031). A full-``N`` ``filtering_bit_mask``
   ``[B, ceil(N / 64)]`` int64 drops a position ``d`` whose bit is clear; the
   CUDA scorer reads bit ``63 - d % 64`` of word ``d // 64`` (high bit first:
   silvertorch/ops/csrc/bloom_index_util.cuh:138-147, 157-180;
   retrieve/src/retrieve/ops/official/__init__.py:31). The exact clause filter
   (``exact_pass``, fork_filters.cuh:15-41, on the layout of ``exact_layout``)
   drops the positions whose clauses fail. Dropped slots are never returned.
4. Top-k on the raw scores, larger first, ties to the lower slot
   (fork_search_cuda.cu:1374-1480; retrieve/src/retrieve/ops/official/adapter.py:465-478),
   over ``min(k, width)`` slots, then the ``[B, k]`` epilogue
   (fork_search_cuda.cu:560-591): ``id = sort_perm[position]``;
   int32 path ``score = fp32(fp32(fp32(dot) * q_scale) * global_scale)``;
   fp16 path ``score = fp32(raw) * fp32(fp32(q_scale * divisor) * global_scale)``
   (adapter.py:363-367, the same left-associated multiplies); ``-1`` / ``-inf``
   past the candidates.

The reference's own check of the op is "scores bit-identical, ids equal up to
ties" against a per-row torch oracle (retrieve/tests/parity/test_official.py:128-160,
211-217). This restatement is pinned to the reference's CPU scorer
(``st.fused_kmean_ann``) and its adapter epilogue (``official_probe_score``) by
``tests/golden/make_golden_ivf.py``.
"""

from __future__ import annotations

import numpy as np

from oracle.knn import quantize_int8

WARP = 32
INT32_MIN = np.iinfo(np.int32).min


def padded_width(max_tensor_size_per_row: int) -> int:
    """retrieve/src/retrieve/ops/official/adapter.py:655-657."""
    return (int(max_tensor_size_per_row) + WARP - 1) // WARP * WARP


def default_divisor(d: int) -> int:
    """Smallest power of two ``v`` with ``127^2 * d / v <= 65504``
    (adapter.py:30-35): the fp16 path's divisor, exact and overflow-free."""
    need = (127 * 127 * d) / 65504.0
    v = 1
    while v < need:
        v *= 2
    return v


def probe_slots(probe_row, cluster_offsets, cluster_sizes) -> np.ndarray:
    """The sorted-table positions one query row scores, in the scorer's slot
    order: warp-aligned prefixes of the probed clusters, then their remainders."""
    heads, tails = [], []
    for c in np.asarray(probe_row, dtype=np.int64).tolist():
        start = int(cluster_offsets[c])
        n = int(cluster_sizes[c])
        full = n // WARP * WARP
        heads.append(np.arange(start, start + full, dtype=np.int64))
        tails.append(np.arange(start + full, start + n, dtype=np.int64))
    return np.concatenate(heads + tails) if heads else np.zeros(0, dtype=np.int64)


def mask_bit_high_first(words_row, pos) -> np.ndarray:
    """Bit of sorted position ``pos`` in one packed ``filtering_bit_mask`` row:
    bit ``63 - pos % 64`` of word ``pos // 64``."""
    w = np.asarray(words_row, dtype=np.int64).view(np.uint64)
    shift = (63 - pos % 64).astype(np.uint64)
    return ((w[pos // 64] >> shift) & np.uint64(1)).astype(bool)


def pack_mask_high_first(mask) -> np.ndarray:
    """``[B, N]`` bool to ``[B, ceil(N / 64)]`` int64, position ``d`` at bit
    ``63 - d % 64`` of word ``d // 64`` (adapter.py:254-267, ``high_first``)."""
    mask = np.asarray(mask, dtype=bool)
    b, n = mask.shape
    w = (n + 63) // 64
    padded = np.zeros((b, w * 64), dtype=bool)
    padded[:, :n] = mask
    bits = padded.reshape(b, w, 64).astype(np.uint64)
    shifts = (63 - np.arange(64)).astype(np.uint64)
    return np.bitwise_or.reduce(bits << shifts, axis=2).view(np.int64)


INT32_MAX = np.iinfo(np.int32).max


def exact_layout(attrs):
    """``[N, C, A]`` cluster-sorted attrs (values ``>= -1``, ``-1`` pads) to the exact
    filter's layout (retrieve/src/retrieve/ops/official/adapter.py:68-81): ``slots``
    int32 ``[R, N]``, clause ``c`` in rows ``clause_slots[c]:clause_slots[c + 1]``,
    each doc's values sorted descending, every clause as wide as its widest doc."""
    a = -np.sort(-np.asarray(attrs, dtype=np.int64), axis=2)  # descending
    if a.size and (a.min() < -1 or a.max() > INT32_MAX):
        raise ValueError("the exact filter takes attr values in [-1, 2**31 - 1]")
    widths = (a != -1).sum(axis=2).max(axis=0) if a.shape[0] else np.zeros(a.shape[1], dtype=np.int64)
    rows = [a[:, c, :w].T for c, w in enumerate(widths.tolist())]
    slots = np.concatenate(rows, axis=0) if rows else np.zeros((0, a.shape[0]), dtype=np.int64)
    clause_slots = np.zeros(a.shape[1] + 1, dtype=np.int64)
    clause_slots[1:] = np.cumsum(widths)
    return np.ascontiguousarray(slots.astype(np.int32)), clause_slots


def exact_query(query_clause_attrs):
    """``[B, C]`` query attrs to int32; a value no doc can hold becomes INT32_MIN
    (adapter.py:84-89)."""
    q = np.asarray(query_clause_attrs, dtype=np.int64)
    return np.where((q >= -1) & (q <= INT32_MAX), q, INT32_MIN).astype(np.int32)


def exact_pass(slots, clause_slots, reverse, q_row, pos) -> np.ndarray:
    """The exact clause test of sorted positions ``pos`` for one query row
    (silvertorch/ops/csrc/fork_filters.cuh:15-41): a clause with query value -1
    passes; otherwise it matches when one of the doc's values equals the query's,
    and passes when the match differs from its reverse flag."""
    slots = np.asarray(slots, dtype=np.int64)
    ok = np.ones(len(pos), dtype=bool)
    for c in range(len(clause_slots) - 1):
        qv = int(q_row[c])
        if qv == -1:
            continue
        vals = slots[clause_slots[c] : clause_slots[c + 1]][:, pos]  # [width, len(pos)]
        match = (vals == qv).any(axis=0)
        ok &= match != bool(reverse[c])
    return ok


def raw_scores(q_codes_row, item_codes, pos, divisor: int):
    """Per-slot raw scores: int32 dots, or fp16 ``dot / divisor``."""
    dots = np.asarray(item_codes, dtype=np.int8)[pos].astype(np.int64) @ np.asarray(q_codes_row, np.int64)
    if divisor == -1:
        return dots.astype(np.int32)
    return (dots.astype(np.float32) / np.float32(divisor)).astype(np.float16)


def search_codes(q_codes, q_scales, probe_ids, cluster_offsets, cluster_sizes, item_codes, sort_perm,
                 global_scale, k, max_tensor_size_per_row, divisor_for_int8=-1, filtering_bit_mask=None,
                 exact=None):
    """``st::search`` after the query prep: ``(ids int64 [B, k], scores fp32 [B, k])``.
    ``exact`` = ``(slots, clause_slots, reverse, query_attrs)`` in the exact filter's
    layout (``exact_layout`` / ``exact_query``) drops the probed positions that fail it."""
    q_codes = np.asarray(q_codes, dtype=np.int8)
    q_scales = np.asarray(q_scales, dtype=np.float32)
    probe_ids = np.asarray(probe_ids, dtype=np.int64)
    offsets = np.asarray(cluster_offsets, dtype=np.int64)
    sizes = np.asarray(cluster_sizes, dtype=np.int64)
    sort_perm = np.asarray(sort_perm, dtype=np.int64)
    gs = np.float32(np.asarray(global_scale, dtype=np.float32).reshape(-1)[0])
    width = padded_width(max_tensor_size_per_row)
    b = q_codes.shape[0]
    ids = np.full((b, k), -1, dtype=np.int64)
    scores = np.full((b, k), -np.inf, dtype=np.float32)
    for row in range(b):
        pos = probe_slots(probe_ids[row], offsets, sizes)
        if pos.size > width:
            raise ValueError(f"row {row} probes {pos.size} positions > width {width}")
        raw = raw_scores(q_codes[row], item_codes, pos, divisor_for_int8)
        slot = np.arange(pos.size, dtype=np.int64)
        if filtering_bit_mask is not None:
            keep = mask_bit_high_first(np.asarray(filtering_bit_mask)[row], pos)
            pos, raw, slot = pos[keep], raw[keep], slot[keep]
        if exact is not None:
            keep = exact_pass(exact[0], exact[1], exact[2], np.asarray(exact[3])[row], pos)
            pos, raw, slot = pos[keep], raw[keep], slot[keep]
        # larger raw first, ties to the lower slot; only min(k, width) slots are taken
        order = np.lexsort((slot, -raw.astype(np.float64)))[: min(k, width)]
        n = order.size
        ids[row, :n] = sort_perm[pos[order]]
        top = raw[order]
        if divisor_for_int8 == -1:
            s = (top.astype(np.float32) * q_scales[row]).astype(np.float32) * gs
        else:
            f = (q_scales[row] * np.float32(divisor_for_int8)).astype(np.float32) * gs
            s = top.astype(np.float32) * np.float32(f)
        scores[row, :n] = s.astype(np.float32)
    return ids, scores


def search(query, probe_ids, cluster_offsets, cluster_sizes, item_codes, sort_perm, global_scale, k,
           max_tensor_size_per_row, divisor_for_int8=-1, filtering_bit_mask=None, exact=None):
    """``st::search`` (fork_search.cpp:13-41) on fp32 queries ``[B, D]``."""
    q_codes, q_scales = quantize_int8(np.asarray(query, dtype=np.float32))
    return search_codes(q_codes, q_scales, probe_ids, cluster_offsets, cluster_sizes, item_codes, sort_perm,
                        global_scale, k, max_tensor_size_per_row, divisor_for_int8, filtering_bit_mask, exact)


FLOAT_PADS = {"fp32": np.float32(-np.finfo(np.float32).max), "fp16": np.float16(-65504.0),
              "bf16": np.uint32(0xFF7F0000).view(np.float32)}


def fused_kmean_ann(q_codes, cluster_offsets, cluster_ids, cluster_length, item_codes, max_tensor_size_per_row,
                    divisor_for_int8=-1, filtering_bit_mask=None, invalid_index_value=-1, partial=None,
                    filtering_bit_index=None, per_embedding_scale=None, float_format=None):
    """``st::fused_kmean_ann`` on int8 codes as its CUDA impl returns it
    (silvertorch/ops/csrc/fused_kmean_ann_cuda.cu:2126-2262, outputs pre-filled at
    :1491-1510): ``(raw [B, W], idx [B, W] int32)``, ``W = padded_width(...)``. Row ``b``
    holds its probes' positions in the slot order of ``probe_slots`` (lengths
    ``cluster_length[b, j]``, not the cluster table's), clipped to ``W`` slots; a slot
    holds the raw score (int32 dot, or fp16 ``dot / divisor``) and the int32 position,
    or ``INT32_MIN`` / fp16 ``-65504`` (``0xfbff``, simple_index_mm.cuh:100-101) and
    ``invalid_index_value`` where nothing was scored: past the row's positions, and where
    the high-bit-first ``filtering_bit_mask`` bit is clear. ``partial`` = ``(cumsum, first,
    words)`` is ``fused_kmean_ann_with_partial_masks``' filter (``partial_mask_keep`` per doc
    of each probed range). ``filtering_bit_index`` [B] maps row ``b`` to the mask row (and the
    partial masks' row) it reads. ``per_embedding_scale`` (fp16 [N], a per-doc divisor that
    takes the divisor's place) gives the fp16 raw ``fp16(fp32(fp16(dot)) / fp32(scale[pos]))``,
    the CUDA scorer's order (index_mm_helpers.cuh:49-56: the dot rounded to fp16 first; the CPU
    scorer divides the unrounded dot, fused_kmean_ann.cpp:196-199, equal for |dot| <= 2048).
    ``float_format`` ("fp32", "fp16", "bf16"; embeddings and queries given as float arrays of
    values in that format) scores by the CUDA scorer's chains (``oracle.fdot.dot``): raw of the
    format (bf16 values as float32), pads -FLT_MAX / -65504 / bf16 0xff7f; no divisor or scale."""
    if float_format is not None:
        return _fused_float(q_codes, cluster_offsets, cluster_ids, cluster_length, item_codes,
                            max_tensor_size_per_row, float_format, filtering_bit_mask, invalid_index_value,
                            filtering_bit_index)
    q_codes = np.asarray(q_codes, dtype=np.int8)
    offsets = np.asarray(cluster_offsets, dtype=np.int64)
    cids = np.asarray(cluster_ids, dtype=np.int64)
    clen = np.asarray(cluster_length, dtype=np.int64)
    n = np.asarray(item_codes).shape[0]
    width = padded_width(max_tensor_size_per_row)
    b = q_codes.shape[0]
    scale = None if per_embedding_scale is None else np.asarray(per_embedding_scale, dtype=np.float16)
    half = divisor_for_int8 != -1 or scale is not None
    raw = np.full((b, width), np.float16(-65504.0) if half else INT32_MIN,
                  dtype=np.float16 if half else np.int32)
    idx = np.full((b, width), invalid_index_value, dtype=np.int32)
    p = cids.shape[1] if cids.ndim == 2 else 0
    rows = np.arange(b) if filtering_bit_index is None else np.asarray(filtering_bit_index, dtype=np.int64)
    for row in range(b):
        heads, tails, keep_h, keep_t = [], [], [], []
        for j, (c, length) in enumerate(zip(cids[row].tolist(), clen[row].tolist())):
            if not 0 <= c < offsets.size - 1 or not 0 <= offsets[c] < n or length <= 0:
                continue
            start = int(offsets[c])
            length = min(length, n - start, width)
            full = length // WARP * WARP
            heads.append(np.arange(start, start + full, dtype=np.int64))
            tails.append(np.arange(start + full, start + length, dtype=np.int64))
            if partial is not None:
                keep = partial_mask_keep(*partial, rows[row] * p + j, np.arange(length))
                keep_h.append(keep[:full])
                keep_t.append(keep[full:])
        pos = np.concatenate(heads + tails)[:width] if heads else np.zeros(0, dtype=np.int64)
        slot = np.arange(pos.size)
        if partial is not None and heads:
            keep = np.concatenate(keep_h + keep_t)[:width]
            pos, slot = pos[keep], slot[keep]
        if filtering_bit_mask is not None:
            keep = mask_bit_high_first(np.asarray(filtering_bit_mask)[rows[row]], pos)
            pos, slot = pos[keep], slot[keep]
        if scale is not None:
            dots = raw_scores(q_codes[row], item_codes, pos, -1)
            raw[row, slot] = (dots.astype(np.float32).astype(np.float16).astype(np.float32)
                              / scale[pos].astype(np.float32)).astype(np.float16)
        else:
            raw[row, slot] = raw_scores(q_codes[row], item_codes, pos, divisor_for_int8)
        idx[row, slot] = pos.astype(np.int32)
    return raw, idx


def _fused_float(q, cluster_offsets, cluster_ids, cluster_length, items, max_tensor_size_per_row, fmt,
                 filtering_bit_mask, invalid_index_value, filtering_bit_index):
    from oracle import fdot

    items = np.asarray(items, dtype=np.float64)
    q = np.asarray(q, dtype=np.float64)
    # the slot layout and the filters of the int8 restatement, on stand-in codes
    zeros = np.zeros(items.shape, dtype=np.int8)
    _, idx = fused_kmean_ann(np.zeros(q.shape, dtype=np.int8), cluster_offsets, cluster_ids, cluster_length, zeros,
                             max_tensor_size_per_row, filtering_bit_mask=filtering_bit_mask,
                             invalid_index_value=-1, filtering_bit_index=filtering_bit_index)
    out_dtype = np.float16 if fmt == "fp16" else np.float32
    raw = np.full(idx.shape, fdot_pad(fmt), dtype=out_dtype)
    for b, s in zip(*np.nonzero(idx >= 0)):
        raw[b, s] = fdot.dot(items[idx[b, s]], q[b], fmt)
    return raw, np.where(idx >= 0, idx, invalid_index_value).astype(np.int32)


def fdot_pad(fmt):
    return FLOAT_PADS[fmt]


def probe_prep(query, probe_ids, cluster_offsets, cluster_sizes):
    """``st::probe_prep`` (fork_search.cpp:43-49; fork_search_cuda.cu:1529-1546): the
    nine outputs the reference checks (retrieve/tests/parity/test_official.py:676-697):
    int8 codes, scales, probed cluster ids, their lengths and offsets, the warp
    count of each (row, probe) flattened, the per-row cumsum of warp-rounded
    lengths, and the global cumsums of remainders and of warp counts."""
    codes, scales = quantize_int8(np.asarray(query, dtype=np.float32))
    probe = np.asarray(probe_ids, dtype=np.int64)
    sizes = np.asarray(cluster_sizes, dtype=np.int64)
    offsets = np.asarray(cluster_offsets, dtype=np.int64)
    length = sizes[probe]
    warps = (length // WARP).astype(np.int32).reshape(-1)
    rounded_cumsum = np.cumsum((warps * WARP).reshape(probe.shape), axis=1, dtype=np.int32)
    rem_cumsum = np.cumsum((length % WARP).reshape(-1), dtype=np.int32)
    warp_cumsum = np.cumsum(warps, dtype=np.int32)
    return codes, scales, probe, length, offsets[probe], warps, rounded_cumsum, rem_cumsum, warp_cumsum


# ---------------------------------------------------------------------------
# SilverTorch's bloom filter (the ``plans`` of st::search without the exact recheck)
# ---------------------------------------------------------------------------
BUNDLE_COLUMNS = 32  # 64-doc columns per bundle: 2048 docs (silvertorch bloom_index_util.h:44-46)
OP_AND, OP_OR, OP_NOT, OP_TERM, OP_EMPTY = 1, 2, 3, 4, 5  # bloom_index_util.h:50-57


def decode_plan(data, offsets, p):
    """Plan ``p`` of the parser's encoding (bloom_index_util.cpp:82-125): eight byte
    offsets per plan into ``data``, giving its operators (uint8), the operators'
    parameter offsets (int32), the parameters (int32) and the terms' stored hashes
    (uint64, ``hash_k`` a term)."""
    raw = np.asarray(data).view(np.uint8)
    o = np.asarray(offsets, dtype=np.int64)[8 * p : 8 * p + 8]
    ops = raw[o[0] : o[1]].copy()
    op_offsets = raw[o[2] : o[3]].copy().view(np.int32)
    hashes = raw[o[6] : o[7]].copy().view(np.uint64)
    return ops, op_offsets, hashes


def plan_blob(data, offsets, slots):
    """The prepared-plan blob st::search reads (adapter.py:212-236): int64 words, the
    parser's eight offsets of each plan first (``8 * slots`` words), then the data."""
    offsets = np.asarray(offsets, dtype=np.int64)
    raw = np.asarray(data).view(np.uint8)
    words = 8 * slots + (len(raw) + 7) // 8
    blob = np.zeros(words, dtype=np.int64)
    blob[: len(offsets)] = offsets
    blob.view(np.uint8)[8 * 8 * slots : 8 * 8 * slots + len(raw)] = raw
    return blob


def bloom_plan_mask(bloom_index, bundle_b_offsets, data, offsets, p, k, hash_k, n):
    """Docs ``[0, n)`` passing plan ``p`` (bloom_index_search_cuda.cu:304-349, 469-544):
    per 64-doc column word, a term ANDs the index rows of its first ``k`` distinct
    positions ``hash % B`` among its ``hash_k`` stored hashes (``B`` the bits of the
    doc's 2048-doc bundle); the operators run as a postfix stack (AND / OR over as many
    children as their parameter range holds, NOT, EMPTY = all); doc ``d`` is bit
    ``63 - d % 64`` of its column's word."""
    index = np.asarray(bloom_index, dtype=np.int64).view(np.uint64)
    boff = np.asarray(bundle_b_offsets, dtype=np.int64)
    ops, op_offsets, hashes = decode_plan(data, offsets, p)
    n_cols = (n + 63) // 64
    cols = np.arange(n_cols)
    bundle = cols // BUNDLE_COLUMNS
    b0 = boff[bundle]
    b_bits = (boff[bundle + 1] - b0).astype(np.uint64)
    in_bundle = cols % BUNDLE_COLUMNS
    full = np.uint64(0xFFFFFFFFFFFFFFFF)

    def term_words(t):
        h = hashes[t * hash_k : (t + 1) * hash_k]
        out = np.full(n_cols, full, dtype=np.uint64)
        for ci in range(n_cols):
            used = []
            for x in h:
                if len(used) == k:
                    break
                pos = int(x % b_bits[ci])
                if pos not in used:
                    used.append(pos)
            w = full
            for pos in used:
                w &= index[(b0[ci] + pos) * BUNDLE_COLUMNS + in_bundle[ci]]
            out[ci] = w
        return out

    stack = []
    term = 0
    for j, op in enumerate(ops.tolist()):
        if op == OP_TERM:
            stack.append(term_words(term))
            term += 1
        elif op in (OP_AND, OP_OR):
            children = int(op_offsets[j + 1] - op_offsets[j])
            acc = np.full(n_cols, full if op == OP_AND else 0, dtype=np.uint64)
            for _ in range(children):
                acc = (acc & stack.pop()) if op == OP_AND else (acc | stack.pop())
            stack.append(acc)
        elif op == OP_NOT:
            stack.append(~stack.pop())
        elif op == OP_EMPTY:
            stack.append(np.full(n_cols, full, dtype=np.uint64))
    words = stack.pop()
    d = np.arange(n)
    return ((words[d // 64] >> (np.uint64(63) - (d % 64).astype(np.uint64))) & np.uint64(1)).astype(bool)


def bloom_full_words(bloom_index, bundle_b_offsets, data, offsets, k, hash_k):
    """``st.bloom_index_search_batch(..., return_bool_mask=False)``
    (bloom_index_search.cpp:178-241): plan ``q`` over every 64-doc column of the index,
    ``[Q, n_bundles * 32]`` int64, doc ``64 c + i`` at bit ``63 - i``."""
    n_docs = (len(bundle_b_offsets) - 1) * BUNDLE_COLUMNS * 64
    q = len(offsets) // 8
    masks = np.stack([bloom_plan_mask(bloom_index, bundle_b_offsets, data, offsets, p, k, hash_k, n_docs)
                      for p in range(q)]) if q else np.zeros((0, n_docs), dtype=bool)
    return pack_mask_high_first(masks)


def column_info(selected_cluster_offsets, selected_cluster_lengths):
    """``st.generate_column_info_for_clusters`` (bloom_index_search.cpp:494-538) for
    non-negative starts: per range the column count ``ceil((length + start % 64) / 64)`` (0 for
    ``length <= 0``), the first column ``start // 64`` and the bit offset ``start % 64``."""
    start = np.asarray(selected_cluster_offsets, dtype=np.int64).reshape(-1)
    length = np.asarray(selected_cluster_lengths, dtype=np.int64).reshape(-1)
    first = start % 64
    counts = np.where(length > 0, (length + first + 63) // 64, 0)
    return counts.astype(np.int32), (start // 64).astype(np.int32), first.astype(np.int8)


def bloom_partial_response(bloom_index, bundle_b_offsets, data, offsets, selected_cluster_offsets,
                           selected_cluster_lengths, k, hash_k, query_plan_index=None):
    """``st.bloom_index_search_batch_return_partial_response`` (bloom_index_search.cpp:244-374):
    ``(column_counts_cumsum int32 [B P], first_item_offset_in_column int8 [B P],
    column_mask_response int64 [total])`` — range after range (row-major over ``[B, P]``), the
    full search's words of the range's columns, row ``b`` running plan
    ``query_plan_index[b]`` (or ``b``)."""
    full = bloom_full_words(bloom_index, bundle_b_offsets, data, offsets, k, hash_k)
    sel = np.asarray(selected_cluster_offsets, dtype=np.int64)
    counts, starts, first = column_info(sel, selected_cluster_lengths)
    b, p = sel.shape
    plans = np.arange(b) if query_plan_index is None else np.asarray(query_plan_index, dtype=np.int64)
    words = [full[plans[i // p], starts[i] : starts[i] + counts[i]] for i in range(b * p)]
    resp = np.concatenate(words) if words else np.zeros(0, dtype=np.int64)
    return np.cumsum(counts, dtype=np.int32), first, resp.astype(np.int64)


def partial_mask_keep(cumsum, first, words, idx, i):
    """Whether ``fused_kmean_ann_with_partial_masks`` keeps doc ``i`` of range ``idx``
    (fused_kmean_ann_cuda.cu:661-721, 800-845): bit ``first[idx] + i`` of the words from
    ``cumsum[idx - 1]`` on, high bit first; a bit past the words drops the doc."""
    base = 0 if idx == 0 else int(cumsum[idx - 1])
    bit = int(first[idx]) + np.asarray(i, dtype=np.int64)
    w = base + bit // 64
    words = np.asarray(words, dtype=np.int64).view(np.uint64)
    ok = w < words.size
    out = np.zeros(np.shape(bit), dtype=bool)
    shift = (63 - bit[ok] % 64).astype(np.uint64)
    out[ok] = ((words[w[ok]] >> shift) & np.uint64(1)).astype(bool)
    return out


def attrs_to_features(attrs):
    """``[N, C, A]`` attrs (``-1`` pads) to the jagged feature layout
    (retrieve/src/retrieve/ops/official/adapter.py:45-65): feature ids ``0 .. C-1``
    int32, CSR offsets over (doc, feature) int64 ``[N C + 1]``, values in (doc,
    feature, slot) order."""
    a = np.asarray(attrs, dtype=np.int64)
    n, c, _ = a.shape
    valid = a != -1
    offsets = np.zeros(n * c + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(valid.sum(axis=2).reshape(-1))
    return np.arange(c, dtype=np.int32), offsets, a.reshape(-1)[valid.reshape(-1)]


def bloom_index_build(feature_ids, feature_offsets, feature_values, b_multiplier, k, bits_per_doc=0):
    """SilverTorch's bundle-major bloom index (silvertorch/ops/csrc/bloom_indexer.cpp:26-114;
    the fixed width of bloom_indexer_cuda.cu:330-335): per 2048-doc bundle ``B`` bits a doc
    (``bits_per_doc``, or ``trunc(fp64(max values of a doc * k) * b_multiplier)``), and for
    every value of feature ``f`` of doc ``d`` its first ``k`` distinct positions
    ``murmur3(f, value, seed) % B`` set bit ``63 - d % 64`` of word
    ``(bundle_b_offsets[d // 2048] + p) * 32 + (d % 2048) // 64``. Returns
    ``(bloom_index int64, bundle_b_offsets int64)``."""
    from oracle.bloom import build_positions

    fid = np.asarray(feature_ids, dtype=np.int64)
    off = np.asarray(feature_offsets, dtype=np.int64)
    val = np.asarray(feature_values, dtype=np.int64)
    c = len(fid)
    n = (len(off) - 1) // c
    n_bundles = (n + 2047) // 2048
    per_doc = off[c::c] - off[: n * c : c]  # values of each doc
    widths = np.zeros(n_bundles, dtype=np.int64)
    for i in range(n_bundles):
        m = int(per_doc[i * 2048 : (i + 1) * 2048].max()) if n else 0
        widths[i] = bits_per_doc if bits_per_doc > 0 else int(float(m * k) * b_multiplier)
    boff = np.zeros(n_bundles + 1, dtype=np.int64)
    boff[1:] = np.cumsum(widths)
    index = np.zeros(int(boff[-1]) * 32, dtype=np.uint64)
    for d in range(n):
        bundle, col = d // 2048, (d % 2048) // 64
        bit = np.uint64(1) << np.uint64(63 - d % 64)
        for f in range(c):
            for v in val[off[d * c + f] : off[d * c + f + 1]]:
                for p in build_positions(int(fid[f]), int(v), int(widths[bundle]), k):
                    index[(boff[bundle] + p) * 32 + col] |= bit
    return index.view(np.int64), boff


# ---------------------------------------------------------------------------
# Row-sharded IVF search: a rank holds the positions [pos_lo, pos_hi) (whole
# clusters), scores them in the global slot layout and returns (raw, slot) pairs;
# the pairs of all ranks merge by (raw desc, slot asc) — the single-GPU tie order —
# and the merged slots map back to positions through the global layout.
# ---------------------------------------------------------------------------
def search_shard(query, probe_ids, cluster_offsets, cluster_sizes, codes_local, pos_lo, k, max_tensor_size_per_row,
                 divisor_for_int8=-1, filtering_bit_mask=None, exact=None):
    """One rank's part: ``(raw [B, k'], slot [B, k'])`` of its best in-window positions
    (``k' = min(k, width)``, ``-inf`` / ``-1`` pads); ``codes_local`` holds the rows
    ``pos_lo ..`` of the sorted table."""
    q_codes, _ = quantize_int8(np.asarray(query, dtype=np.float32))
    probe_ids = np.asarray(probe_ids, dtype=np.int64)
    codes_local = np.asarray(codes_local, dtype=np.int8)
    pos_hi = pos_lo + codes_local.shape[0]
    width = padded_width(max_tensor_size_per_row)
    k_sel = min(k, width)
    b = q_codes.shape[0]
    raw_out = np.full((b, k_sel), -np.inf, dtype=np.float64)
    slot_out = np.full((b, k_sel), -1, dtype=np.int64)
    for row in range(b):
        pos = probe_slots(probe_ids[row], cluster_offsets, cluster_sizes)
        slot = np.arange(pos.size, dtype=np.int64)
        keep = (pos >= pos_lo) & (pos < pos_hi) & (slot < width)
        if filtering_bit_mask is not None:
            keep &= mask_bit_high_first(np.asarray(filtering_bit_mask)[row], pos)
        if exact is not None:
            keep &= exact_pass(exact[0], exact[1], exact[2], np.asarray(exact[3])[row], pos)
        pos, slot = pos[keep], slot[keep]
        raw = raw_scores(q_codes[row], codes_local, pos - pos_lo, divisor_for_int8).astype(np.float64)
        order = np.lexsort((slot, -raw))[:k_sel]
        raw_out[row, : order.size] = raw[order]
        slot_out[row, : order.size] = slot[order]
    return raw_out, slot_out


def merge_shards(raws, slots, k):
    """The ranks' pairs to the global best ``k`` by (raw desc, slot asc)."""
    raw = np.concatenate(raws, axis=1)
    slot = np.concatenate(slots, axis=1)
    b = raw.shape[0]
    out_r = np.full((b, k), -np.inf)
    out_s = np.full((b, k), -1, dtype=np.int64)
    for row in range(b):
        ok = slot[row] >= 0
        r, s = raw[row][ok], slot[row][ok]
        order = np.lexsort((s, -r))[:k]
        out_r[row, : order.size] = r[order]
        out_s[row, : order.size] = s[order]
    return out_r, out_s


def finish_shards(query, probe_ids, cluster_offsets, cluster_sizes, sort_perm, global_scale, raw, slot,
                  divisor_for_int8=-1):
    """Merged (raw, slot) to ``(ids, scores)``: the slot's position in the global layout,
    ``sort_perm`` and the epilogue's two multiplies."""
    _, q_scales = quantize_int8(np.asarray(query, dtype=np.float32))
    gs = np.float32(np.asarray(global_scale, dtype=np.float32).reshape(-1)[0])
    sort_perm = np.asarray(sort_perm, dtype=np.int64)
    b, k = raw.shape
    ids = np.full((b, k), -1, dtype=np.int64)
    scores = np.full((b, k), -np.inf, dtype=np.float32)
    for row in range(b):
        pos = probe_slots(np.asarray(probe_ids)[row], cluster_offsets, cluster_sizes)
        for j in range(k):
            if slot[row, j] < 0:
                continue
            ids[row, j] = sort_perm[pos[slot[row, j]]]
            r = np.float32(raw[row, j])
            if divisor_for_int8 == -1:
                scores[row, j] = np.float32(np.float32(r * q_scales[row]) * gs)
            else:
                scores[row, j] = r * np.float32(np.float32(q_scales[row] * np.float32(divisor_for_int8)) * gs)
    return ids, scores
