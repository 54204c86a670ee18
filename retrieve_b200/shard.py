"""Row-sharded search over several GPUs (one process per GPU).

The corpus is split row-wise into contiguous shards; rank ``r`` holds rows
``[offset_r, offset_r + n_r)``. A query batch (replicated on every rank) is
scored against the local shard with the fused kernel. One search is:

1. every rank samples its shard (``dense_seed_sample``: k tile maxima per
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

The two all-gathers run through NCCL (``exchange="nccl"``) or through the peers'
memory (``exchange="peer"``, :class:`PeerExchange`): every rank pushes its block
into every peer's exchange buffer with plain peer stores and raises a flag there,
and reads the stack from its own buffer once every flag is up (one node, CUDA
IPC mappings, no multicast).

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


class PeerExchange:
    """A fixed-size all-gather through the peers' memory on one node
    (``rb_peer_allgather``): ``allgather(t)`` returns the ``[W, *t.shape]`` stack of every
    rank's ``t`` in rank order, in a buffer owned by this object (the next call
    overwrites it). Built collectively (every rank of ``group`` constructs it with the
    same ``slot_bytes``); every rank then calls ``allgather`` the same number of times.
    The step counter lives on the device, so calls captured in a CUDA graph replay."""

    def __init__(self, slot_bytes: int, device: torch.device, group=None) -> None:
        lib = _lib.lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.device = torch.device(device)
        self.slot_bytes = (int(slot_bytes) + 15) // 16 * 16
        nbytes = lib.rb_peer_buffer_bytes(self.world, self.slot_bytes)
        own = ctypes.c_void_p(0)
        handle = (ctypes.c_ubyte * 64)()
        with torch.cuda.device(self.device):
            _lib.check(lib.rb_ipc_alloc(nbytes, ctypes.byref(own), handle), "peer exchange buffer")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        bases, self._opened = [], []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                p = ctypes.c_void_p(0)
                _lib.check(lib.rb_ipc_open((ctypes.c_ubyte * 64).from_buffer_copy(h), ctypes.byref(p)),
                           "peer exchange mapping")
                bases.append(p.value)
                self._opened.append(p.value)
        self._bases = (ctypes.c_void_p * self.world)(*bases)
        # step (int64), push-completion count (int32), error word (int32)
        self._counters = torch.zeros(16, dtype=torch.uint8, device=self.device)
        self._out: Tensor | None = None
        self._stage: Tensor | None = None
        dist.barrier(group=group)  # every buffer is zeroed and mapped before any push

    def allgather(self, t: Tensor) -> Tensor:
        t = t.contiguous()
        nbytes = t.numel() * t.element_size()
        padded = (nbytes + 15) // 16 * 16
        if padded > self.slot_bytes:
            raise ValueError(f"peer exchange: {nbytes} bytes do not fit the {self.slot_bytes}-byte slots")
        src = t
        if padded != nbytes:  # blocks move in 16-byte units: stage the tail
            if self._stage is None or self._stage.numel() != padded:
                self._stage = torch.zeros(padded, dtype=torch.uint8, device=self.device)
            self._stage[:nbytes].copy_(t.view(-1).view(torch.uint8))
            src = self._stage
        if self._out is None or self._out.numel() != self.world * padded:
            self._out = torch.empty((self.world, padded), dtype=torch.uint8, device=self.device)
        c = self._counters.data_ptr()
        rc = _lib.lib().rb_peer_allgather(
            self._bases, self.world, self.rank, self.slot_bytes, ctypes.c_void_p(src.data_ptr()), padded,
            ctypes.c_void_p(c), ctypes.c_void_p(c + 8), ctypes.c_void_p(c + 12), ctypes.c_void_p(self._out.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream),
        )
        _lib.check(rc, "peer allgather")
        stack = self._out if padded == nbytes else self._out[:, :nbytes].contiguous()
        return stack.view(t.dtype).view(self.world, *t.shape)

    def device_error(self) -> int:
        """The error word: 0, or 5 when a peer's flag did not come up within the wait limit."""
        return int(self._counters[12:16].view(torch.int32).item())

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective: no rank may still
        be pushing or reading)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.rb_ipc_close(ctypes.c_void_p(p))
            self._opened = []
            dist.barrier(group=self.group)
            if self._own:
                lib.rb_ipc_free(ctypes.c_void_p(self._own))
                self._own = 0


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

    def __init__(self, item_shard: Tensor, id_offset: int, k: int, group=None, n_total: int | None = None,
                 exchange: str = "nccl") -> None:
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be 'nccl' or 'peer', got {exchange!r}")
        self.exchange = exchange
        self._peer: dict[str, PeerExchange] = {}
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
        # each shard sends its top m sampled tile maxima per query: any subset
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
        gathered = self._allgather("samples", vals)
        pairs = ops.dense_topk_seeded(
            query, self.items, self.k, self.id_offset, self.n_total, gathered.view(self.world, b, m), ws,
            pairs=True,
        )
        all_pairs = self._allgather("pairs", pairs)
        return ops.merge_pairs(all_pairs.view(self.world, b, self.k), self.k)

    def _allgather(self, what: str, t: Tensor) -> Tensor:
        """``[W, *t.shape]`` stack of every rank's ``t`` (NCCL, or the peers' memory)."""
        if self.exchange == "nccl":
            out = torch.empty((self.world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
            return out.view(self.world, *t.shape)
        nbytes = t.numel() * t.element_size()
        ex = self._peer.get(what)
        if ex is None or ex.slot_bytes < nbytes:  # built at the first (eager) search, collectively
            if ex is not None:
                ex.close()
            ex = PeerExchange(nbytes, t.device, self.group)
            self._peer[what] = ex
        return ex.allgather(t)

    def close(self) -> None:
        """Releases the peer exchange buffers (collective)."""
        for ex in self._peer.values():
            ex.close()
        self._peer = {}

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
        sampled = n.value >= 4
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
