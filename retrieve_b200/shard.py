"""Row-sharded search over several GPUs (one process per GPU).

The corpus is split row-wise into contiguous shards; rank ``r`` holds rows
``[offset_r, offset_r + n_r)``. A query batch (replicated on every rank) is
scored against the local shard with the fused kernel. One search is:

1. every rank samples its shard (``dense_seed_sample``: k chunk maxima per
   query) and one NCCL all-gather brings the ``[W, B, k]`` samples to every rank;
2. every rank runs the full pass over its shard seeded by the k-th largest
   value of the union — a lower bound on the global k-th score — and keeps its
   local top-k as packed (score, global id) pairs;
3. a second all-gather brings the ``[W, B, k]`` pairs to every rank and
   ``merge_pairs`` reduces them to the global top-k with the single-GPU ordering
   (score descending, ties to the lower id).

Exact for any ``W``: the global top-k is contained in the union of the local
top-k lists (the shared seed never drops a global top-k item), and a shard's
scores do not depend on which shard scores it.

The reference is single-GPU (its harness merges chunked top-k lists the same
way on one device, evaluation/bench/oracle.py:83-92); this module is the
multi-GPU extension of ``PostfilterKNN`` (retrieve/src/retrieve/modules/knn.py:23-76).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
from torch import Tensor

from retrieve_b200 import _lib, ops


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """``[start, end)`` rows of shard ``rank`` of an ``n``-row corpus."""
    return (n * rank) // world, (n * (rank + 1)) // world


def merge_topk(ids: Tensor, scores: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """``[W, B, kin]`` per-shard results → global ``[B, k]`` (C-ABI ``rb_merge_topk``)."""
    if ids.dim() != 3 or ids.shape != scores.shape:
        raise ValueError("ids and scores must both be [W, B, kin]")
    ids = ids.contiguous()
    scores = scores.to(torch.float32).contiguous()
    w, b, kin = ids.shape
    dev = ids.device
    out_i = torch.empty((b, k), dtype=torch.int64, device=dev)
    out_s = torch.empty((b, k), dtype=torch.float32, device=dev)
    lib = _lib.lib()
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_merge_topk_workspace_size(w, b, kin, ctypes.byref(nb)), "merge_topk")
    ws = torch.empty(max(int(nb.value), 256), dtype=torch.uint8, device=dev)
    rc = lib.rb_merge_topk(
        ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(scores.data_ptr()), w, b, kin, k,
        ctypes.c_void_p(out_i.data_ptr()), ctypes.c_void_p(out_s.data_ptr()),
        ctypes.c_void_p(ws.data_ptr()), ws.numel(),
        ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream),
    )
    _lib.check(rc, "merge_topk")
    return out_i, out_s


def exchange_and_merge(ids: Tensor, scores: Tensor, k: int, group=None, merge=None) -> tuple[Tensor, Tensor]:
    """The exchange step of a row-sharded search: all-gather every rank's local
    ``[B, k]`` (ids already global) and reduce the ``[W, B, k]`` stack to the
    global top-k with ``merge`` (default: the CUDA merge kernel). Every rank
    takes the same collective steps in the same order."""
    world = dist.get_world_size(group)
    b, kin = ids.shape
    all_i = torch.empty((world * b, kin), dtype=ids.dtype, device=ids.device)
    all_s = torch.empty((world * b, kin), dtype=scores.dtype, device=scores.device)
    dist.all_gather_into_tensor(all_i, ids.contiguous(), group=group)
    dist.all_gather_into_tensor(all_s, scores.contiguous(), group=group)
    return (merge or merge_topk)(all_i.view(world, b, kin), all_s.view(world, b, kin), k)


class ShardedDenseTopK:
    """The local shard of a row-sharded dense index plus the exchange steps.

    ``item_shard`` is this rank's ``[n_r, D]`` fp16/bf16 rows (contiguous) and
    ``id_offset`` their first global id; ``n_total`` is the corpus size over all
    ranks (summed over the group when not given: a collective at construction).
    ``search(query)`` returns the global ``(ids [B, k], scores [B, k])`` on every
    rank. With more than one rank the threshold seed is shared: every rank
    samples its shard (``dense_seed_sample``), one all-gather brings the samples
    together, and every rank's full pass starts from the k-th largest value of
    their union — the seed one GPU would take over the whole corpus — so each
    shard appends about 1/W of the candidates a shard-local seed would."""

    def __init__(self, item_shard: Tensor, id_offset: int, k: int, group=None, n_total: int | None = None) -> None:
        ops.check_contiguous(item_shard=item_shard)
        self.items = item_shard
        self.id_offset = int(id_offset)
        self.k = int(k)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if n_total is None:
            n_total = item_shard.shape[0]
            if self.world > 1:
                t = torch.tensor([n_total], dtype=torch.int64, device=item_shard.device)
                dist.all_reduce(t, group=group)
                n_total = int(t.item())
        self.n_total = int(n_total)
        # each shard sends its top m sampled chunk maxima per query: any subset
        # keeps the union's k-th a valid bound, and about 2k/W keeps it as tight
        # as all k unless one shard holds more than m of the global top chunks
        self.sample_width = min(self.k, max(16, -(-2 * self.k // max(self.world, 1))))
        self._ws: Tensor | None = None
        self._ws_batch = 0

    def local(self, query: Tensor) -> tuple[Tensor, Tensor]:
        return ops.dense_topk_sharded(query, self.items, self.k, self.id_offset, self._workspace(query))

    def _workspace(self, query: Tensor) -> Tensor:
        """One persistent device workspace per index (graphs captured from it
        all use the same buffer)."""
        b = query.shape[0]
        if self._ws is None or self._ws_batch < b or self._ws.device != query.device:
            self._ws = ops.dense_workspace(query, self.items, self.k)
            self._ws_batch = b
        return self._ws

    def search(self, query: Tensor) -> tuple[Tensor, Tensor]:
        if self.world == 1:
            return self.local(query)
        ws = self._workspace(query)
        m = self.sample_width
        vals = ops.dense_seed_sample(query, self.items, self.k, self.n_total, ws, m)
        b = vals.shape[0]
        gathered = torch.empty((self.world * b, m), dtype=vals.dtype, device=vals.device)
        dist.all_gather_into_tensor(gathered, vals, group=self.group)
        pairs = ops.dense_topk_seeded(
            query, self.items, self.k, self.id_offset, self.n_total, gathered.view(self.world, b, m), ws,
            pairs=True,
        )
        all_pairs = torch.empty((self.world * b, self.k), dtype=pairs.dtype, device=pairs.device)
        dist.all_gather_into_tensor(all_pairs, pairs, group=self.group)
        return ops.merge_pairs(all_pairs.view(self.world, b, self.k), self.k)

    def launches_per_search(self, b: int) -> int:
        """Kernels of this library one search launches (NCCL's not counted)."""
        lib = _lib.lib()
        n = ctypes.c_int(0)
        _lib.check(
            lib.rb_dense_topk_launches(b, self.items.shape[0], self.items.shape[1], 1, self.k, ctypes.byref(n)),
            "launches",
        )
        if self.world == 1:
            return n.value
        sampled = n.value == 4
        # sample pass + row select (or the -inf fill), union select, full pass,
        # list merge into pairs, then the merge of the gathered pairs
        return (2 if sampled else 1) + 1 + 2 + 1


class GraphedSearch:
    """One search of a fixed query batch shape captured as a CUDA graph.

    Repeated searches of the same batch size replay the captured kernels (and,
    with more than one rank, the NCCL all-gathers) without host launch work.
    ``example`` is a query batch of the shape and dtype to serve; it is used for
    the warm-up searches that precede the capture (communicators, workspace,
    kernel attributes). ``search(query)`` copies ``query`` (host — pinned for an
    asynchronous copy — or device) into the static input, replays, and returns
    the static ``(ids, scores)`` outputs, which the next call overwrites. Every
    rank must construct and call it the same number of times. Graphs given the
    same ``pool`` (``torch.cuda.graph_pool_handle()``) share memory and must
    then be replayed in the order they were made, never concurrently."""

    def __init__(self, index: ShardedDenseTopK, example: Tensor, warmup: int = 2, pool=None) -> None:
        dev = index.items.device
        self.index = index
        self.query = example.to(device=dev, dtype=index.items.dtype).contiguous().clone()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                index.search(self.query)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool):
            self.ids, self.scores = index.search(self.query)
        torch.cuda.synchronize(dev)

    def replay(self) -> tuple[Tensor, Tensor]:
        self.graph.replay()
        return self.ids, self.scores

    def search(self, query: Tensor) -> tuple[Tensor, Tensor]:
        self.query.copy_(query, non_blocking=True)
        return self.replay()

    def release(self) -> None:
        """Drops the graph (before the process group is destroyed)."""
        self.graph.reset()


class ShardedOneBitRerank:
    """Row-sharded LiNR V3 cascade (config 5): 1-bit top-``pool`` candidates,
    then exact rescoring to the top ``k``, with two exchanges.

    1. every rank takes its shard's 1-bit top-``pool`` (global ids, tensor
       cores), one all-gather + merge gives every rank the global pool — the
       single-GPU pool exactly (integer scores, ties to the lower id);
    2. every rank rescores the pool entries it owns (its rows of the fp16/bf16
       table, ``fused_masked_knn_topk``), one all-gather + merge gives the top k.

    ``item_bits`` ``[n_r, W]`` int64 and ``item_embs`` ``[n_r, D]`` are this
    rank's rows, starting at global id ``id_offset``. Stage-2 ties (equal fp32
    scores) between items of different shards go to the lower global id."""

    def __init__(self, item_bits: Tensor, item_embs: Tensor, id_offset: int, pool: int, k: int, group=None) -> None:
        from retrieve_b200.bitknn import PackedBitsIndex

        if k > pool:
            raise ValueError(f"k={k} exceeds candidate_pool={pool}")
        if item_bits.shape[0] != item_embs.shape[0]:
            raise ValueError("item_bits and item_embs must hold the same rows")
        ops.check_contiguous(item_embs=item_embs)
        self.bits = PackedBitsIndex(item_bits)
        self.items = item_embs
        self.id_offset = int(id_offset)
        self.pool = int(pool)
        self.k = int(k)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def _exchange(self, ids: Tensor, scores: Tensor, k: int) -> tuple[Tensor, Tensor]:
        if self.world == 1:
            return ids, scores
        return exchange_and_merge(ids, scores, k, self.group)

    def search(self, query: Tensor, query_bits: Tensor) -> tuple[Tensor, Tensor]:
        ids1, sc1 = self.bits.topk(query_bits, self.pool, self.id_offset)
        pool_ids, _ = self._exchange(ids1, sc1, self.pool)
        # this shard's rows of the pool, as local rows (others fall outside
        # [0, n_r) and are not scored)
        local = pool_ids - self.id_offset
        counts = torch.full((local.shape[0],), local.shape[1], dtype=torch.int64, device=local.device)
        k2 = min(self.k, local.shape[1])
        ids2, sc2 = ops.fused_masked_knn_topk(query, self.items, local, counts, k2)
        ids2 = torch.where(ids2 >= 0, ids2 + self.id_offset, ids2)
        return self._exchange(ids2, sc2, self.k)


def ivf_shard_bounds(cluster_offsets, world: int, rank: int) -> tuple[int, int, int, int]:
    """Rank ``rank``'s share of a cluster-sorted IVF table: clusters ``[c_lo, c_hi)`` and their
    sorted positions ``[pos_lo, pos_hi)``. Whole clusters, cut where the position count
    crosses ``n * r / world``."""
    import bisect

    off = [int(x) for x in (cluster_offsets.tolist() if hasattr(cluster_offsets, "tolist") else cluster_offsets)]
    n, n_lists = off[-1], len(off) - 1

    def cut(r: int) -> int:
        return 0 if r == 0 else n_lists if r == world else bisect.bisect_left(off, (n * r) // world, 0, n_lists)

    c_lo, c_hi = cut(rank), cut(rank + 1)
    return c_lo, c_hi, off[c_lo], off[c_hi]


class ShardedIVFSearch:
    """``st::search`` over a cluster-sorted int8 table split across ranks by whole clusters
    (``ivf_shard_bounds``). Every rank holds its rows ``[pos_lo, pos_hi)`` of the codes and
    the whole table's small tables (cluster offsets and sizes, ``sort_perm``, the filter's
    tables); the query batch and its probe lists are replicated. One search:

    1. every rank scores the probed positions it holds, in the whole table's slot layout, and
       keeps its best ``min(k, width)`` as packed (raw score, slot) pairs (``st.search_shard``);
    2. one all-gather brings the ``[W, B, k']`` pairs to every rank and ``merge_pairs``
       reduces them by (raw descending, slot ascending) — the single-GPU order, ties included;
    3. ``st.search_finish`` maps each slot to its position, id and dequantized score.

    The result equals ``st::search`` on the whole table on one GPU, bit for bit.
    """

    def __init__(self, codes_shard: Tensor, pos_lo: int, cluster_offsets: Tensor, cluster_sizes: Tensor,
                 sort_perm: Tensor, global_scale: Tensor, group=None) -> None:
        self.codes = codes_shard.contiguous()
        self.pos_lo = int(pos_lo)
        self.offsets = cluster_offsets
        self.sizes = cluster_sizes
        self.sort_perm = sort_perm
        self.global_scale = global_scale
        self.n_total = int(sort_perm.numel())
        self.group = group

    def local(self, query: Tensor, probe_ids: Tensor, k: int, width: int, divisor: int, filters: dict) -> Tensor:
        from retrieve_b200 import st

        return st.search_shard(query, probe_ids, self.offsets, self.sizes, self.n_total, self.pos_lo, self.codes, k,
                               width, divisor, **filters)

    def merge(self, stack: Tensor, k: int) -> tuple[Tensor, Tensor]:
        return ops.merge_pairs(stack, k)

    def finish(self, query: Tensor, probe_ids: Tensor, k: int, width: int, slots: Tensor, raw: Tensor,
               divisor: int) -> tuple[Tensor, Tensor]:
        from retrieve_b200 import st

        return st.search_finish(query, probe_ids, self.offsets, self.sizes, self.sort_perm, self.global_scale, k,
                                width, slots, raw, divisor)

    def search(self, query: Tensor, probe_ids: Tensor, k: int, max_tensor_size_per_row: int,
               divisor_for_int8: int = -1, **filters) -> tuple[Tensor, Tensor]:
        pairs = self.local(query, probe_ids, k, max_tensor_size_per_row, divisor_for_int8, filters)
        world = dist.get_world_size(self.group)
        b, kin = pairs.shape
        gathered = torch.empty((world * b, kin), dtype=pairs.dtype, device=pairs.device)
        dist.all_gather_into_tensor(gathered, pairs.contiguous(), group=self.group)
        slots, raw = self.merge(gathered.view(world, b, kin), kin)
        return self.finish(query, probe_ids, k, max_tensor_size_per_row, slots, raw, divisor_for_int8)
