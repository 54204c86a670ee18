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
