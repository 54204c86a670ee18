"""Multi-rank logic of the row-sharded search on CPU (gloo, world size 2 and
3): shard bounds cover the corpus exactly once, every rank's local top-k uses
global ids, and exchange_and_merge (all-gather + merge) returns on every rank
the exact global top-k of the whole corpus. The local top-k and the merge are
the oracle's here (the GPU path plugs in the CUDA kernels)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from retrieve_b200.shard import exchange_and_merge, shard_bounds


def _oracle_merge(all_i, all_s, k):
    from oracle.select import merge_topk

    i, s = merge_topk(list(all_i.numpy()), list(all_s.numpy()), k)
    return torch.from_numpy(i), torch.from_numpy(s)


def _worker(rank, world, port, q, x, k, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from oracle.dense import dense_topk

    lo, hi = shard_bounds(x.shape[0], world, rank)
    li, ls = dense_topk(q, x[lo:hi], k)
    li = np.where(li >= 0, li + lo, -1)
    ids, scores = exchange_and_merge(torch.from_numpy(li), torch.from_numpy(ls), k, merge=_oracle_merge)
    out[rank] = (ids.numpy(), scores.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_merge_equals_global_topk(world):
    g = torch.Generator().manual_seed(world)
    q = torch.randint(-3, 4, (16, 32), generator=g).float().numpy()
    x = torch.randint(-3, 4, (5003, 32), generator=g).float().numpy()
    k = 50
    bounds = [shard_bounds(x.shape[0], world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == x.shape[0]
    assert all(bounds[r][1] == bounds[r + 1][0] for r in range(world - 1))
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    port = 29500 + 7 * world
    mp.start_processes(_worker, args=(world, port, q, x, k, out), nprocs=world, join=True, start_method="spawn")
    from oracle.dense import dense_topk

    ref_i, ref_s = dense_topk(q, x, k)
    for r in range(world):
        ids, scores = out[r]
        assert np.array_equal(scores, ref_s) and np.array_equal(ids, ref_i)


def _pack_pairs(raw, slot):
    """(raw, slot) [B, k] to the packed int64 pairs of rb_st_search_shard (raw score bits low,
    slot high; padding -inf / 0xffffffff)."""
    lo = np.asarray(raw, dtype=np.float32).view(np.uint32).astype(np.uint64)
    hi = np.where(slot >= 0, slot, 0xFFFFFFFF).astype(np.uint64)
    return ((hi << np.uint64(32)) | lo).view(np.int64)


def _unpack_pairs(pairs):
    p = np.asarray(pairs).view(np.uint64)
    raw = (p & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32).astype(np.float64)
    slot = (p >> np.uint64(32)).astype(np.int64)
    return raw, np.where(slot == 0xFFFFFFFF, -1, slot)


def _ivf_worker(rank, world, port, case, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from oracle import ivf
    from retrieve_b200.shard import ShardedIVFSearch, ivf_shard_bounds

    g, k, width, words = case
    _, _, lo, hi = ivf_shard_bounds(g["offsets"], world, rank)

    class OracleShards(ShardedIVFSearch):
        # the host logic of the exchange with the oracle in place of the kernels (CPU ranks)
        def local(self, query, probe_ids, k, width, divisor, filters):
            mask = filters.get("filtering_bit_mask")
            raw, slot = ivf.search_shard(query.numpy(), probe_ids.numpy(), g["offsets"], g["sizes"],
                                         self.codes.numpy(), self.pos_lo, k, width,
                                         filtering_bit_mask=None if mask is None else mask.numpy())
            return torch.from_numpy(_pack_pairs(raw, slot))

        def merge(self, stack, k):
            # (slots, raw), the order of ops.merge_pairs' (ids, scores)
            raws, slots = zip(*(_unpack_pairs(s) for s in stack.numpy()))
            raw, slot = ivf.merge_shards(list(raws), list(slots), k)
            return slot, raw

        def finish(self, query, probe_ids, k, width, slots, raw, divisor):
            ids, scores = ivf.finish_shards(query.numpy(), probe_ids.numpy(), g["offsets"], g["sizes"],
                                            g["sort_perm"], g["gs"], raw, slots)
            return ids, scores

    index = OracleShards(torch.from_numpy(g["codes"][lo:hi]), lo, g["offsets"], g["sizes"],
                         torch.from_numpy(g["sort_perm"]), torch.from_numpy(g["gs"]))
    filters = {} if words is None else {"filtering_bit_mask": torch.from_numpy(words)}
    ids, scores = index.search(torch.from_numpy(g["query"]), torch.from_numpy(g["probe"]), k, width, **filters)
    out[rank] = (ids, scores)
    dist.destroy_process_group()


@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("world", [2, 3])
def test_sharded_ivf_search_equals_single_search(world, masked):
    """Row-sharded st::search (whole clusters a rank): local (raw, slot) pairs in the whole
    table's slot layout, one all-gather, the (raw desc, slot asc) merge and the slot -> id
    finish give the single-table search bit for bit, ties included (the tie-heavy fixture
    case)."""
    from pathlib import Path

    from oracle import ivf

    golden = np.load(Path(__file__).resolve().parent / "golden" / "golden_ivf.npz")
    p = "c6_"
    g = {key[len(p):]: golden[key] for key in golden.files if key.startswith(p)}
    n_lists, max_size, n_probe, d, k, b, width, div, ties = g["shape"].tolist()
    assert ties
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    port = 29700 + 11 * world + (5 if masked else 0)
    words = ivf.pack_mask_high_first(g["mask"]) if masked else None
    mp.start_processes(_ivf_worker, args=(world, port, (g, k, width, words), out), nprocs=world, join=True,
                       start_method="spawn")
    want_i, want_s = ivf.search(g["query"], g["probe"], g["offsets"], g["sizes"], g["codes"], g["sort_perm"],
                                g["gs"], k, width, filtering_bit_mask=words)
    k_sel = min(k, ivf.padded_width(width))
    for r in range(world):
        ids, scores = out[r]
        assert np.array_equal(ids, want_i[:, :k_sel]) and np.array_equal(scores, want_s[:, :k_sel])


def _leaving_worker(rank, world, port, q, x, k, out):
    """Step 1 on every rank; then rank 1 leaves between steps (no collective of step 2
    in flight) and rank 0's step 2 must end with an error from the process group's
    short timeout instead of waiting for good."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import time
    from datetime import timedelta

    # a generous timeout for the rendezvous (process start-up varies), a short one for the steps
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    short = dist.new_group(list(range(world)), timeout=timedelta(seconds=3))
    from oracle.dense import dense_topk

    lo, hi = shard_bounds(x.shape[0], world, rank)
    li, ls = dense_topk(q, x[lo:hi], k)
    li = np.where(li >= 0, li + lo, -1)
    exchange_and_merge(torch.from_numpy(li), torch.from_numpy(ls), k, group=short, merge=_oracle_merge)
    out[f"step1_{rank}"] = True
    if rank == 1:
        time.sleep(8)  # gone for longer than the timeout: never joins step 2
        out["left"] = True
        return
    t0 = time.monotonic()
    try:
        exchange_and_merge(torch.from_numpy(li), torch.from_numpy(ls), k, group=short, merge=_oracle_merge)
        out["step2_0"] = "completed"
    except Exception as exc:  # noqa: BLE001  (the timeout surfaces as a backend-specific error type)
        out["step2_0"] = type(exc).__name__
    out["waited_s"] = time.monotonic() - t0


def test_rank_leaving_between_steps_ends_the_next_exchange_with_an_error():
    g = torch.Generator().manual_seed(5)
    q = torch.randint(-3, 4, (8, 32), generator=g).float().numpy()
    x = torch.randint(-3, 4, (2001, 32), generator=g).float().numpy()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_leaving_worker, args=(2, 29611, q, x, 20, out), nprocs=2, join=True, start_method="spawn")
    assert out["step1_0"] and out["step1_1"] and out["left"]
    assert out["step2_0"] != "completed"
    assert out["waited_s"] < 30.0
