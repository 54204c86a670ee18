"""Row-sharded search with the threshold seed shared by all shards.

The W shards of a corpus run on one GPU here, one after the other, through
exactly the calls a rank makes (``dense_seed_sample`` on its shard, the [W, B, k]
stack an all-gather would build, ``dense_topk_seeded`` on its shard, then the
cross-shard ``merge_topk``). An item's score does not depend on which shard
scores it, so the merged result must equal single-call ``dense_topk`` over the
whole corpus bit for bit — ids and scores, ties to the lower global id. The
multi-rank exchange itself (NCCL / gloo all-gather) is covered by
tests/test_shard_gloo.py on CPU.
"""

from __future__ import annotations

import pytest
import torch

from retrieve_b200 import ops
from retrieve_b200.shard import merge_topk, shard_bounds
from tests.helpers import assert_topk_exact, make_int_rows, mixture_rows

pytestmark = pytest.mark.gpu


def _sharded(q, x, k, bounds, pairs=False, m=None):
    """m = None: the sample width ShardedDenseTopK uses (about 2k/W)."""
    n_total = x.shape[0]
    w = len(bounds)
    m = min(k, max(16, -(-2 * k // w))) if m is None else m
    shards = [x[lo:hi].contiguous() for lo, hi in bounds]
    samples = torch.stack([ops.dense_seed_sample(q, s, k, n_total, m=m) for s in shards])
    if pairs:
        # what a rank exchanges: one [B, k] int64 tensor of (score, id) pairs
        stack = torch.stack(
            [ops.dense_topk_seeded(q, s, k, lo, n_total, samples, pairs=True) for s, (lo, _) in zip(shards, bounds)]
        )
        return ops.merge_pairs(stack, k)
    outs = [ops.dense_topk_seeded(q, s, k, lo, n_total, samples) for s, (lo, _) in zip(shards, bounds)]
    ids = torch.stack([o[0] for o in outs])
    scores = torch.stack([o[1] for o in outs])
    return merge_topk(ids, scores, k)


@pytest.mark.parametrize("pairs,full_width", [(False, True), (True, False), (True, True)])
@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("b,n,k", [(300, 400_003, 100), (1024, 1_000_000, 100), (96, 150_001, 37)])
def test_shared_seed_equals_single_call_integer(world, b, n, k, pairs, full_width):
    q = make_int_rows(b, 128, seed=11, device="cuda")
    x = make_int_rows(n, 128, seed=12, device="cuda")
    ref_i, ref_s = ops.dense_topk(q, x, k)
    bounds = [shard_bounds(n, world, r) for r in range(world)]
    ids, scores = _sharded(q, x, k, bounds, pairs, m=k if full_width else None)
    torch.cuda.synchronize()
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i.cpu().numpy(), ref_s.cpu().numpy())


@pytest.mark.parametrize("world", [2, 8])
def test_shared_seed_equals_single_call_mixture(world):
    # the benchmark's corpus family: clustered, so candidates concentrate
    b, n, k = 1024, 2_000_000, 100
    x, cent = mixture_rows(n, 128, n_centres=1024, sigma=0.15, seed=5, dtype=torch.bfloat16, device="cuda")
    q, _ = mixture_rows(b, 128, n_centres=1024, sigma=0.15, seed=6, dtype=torch.bfloat16, device="cuda",
                        centres=cent)
    ref_i, ref_s = ops.dense_topk(q, x, k)
    ids, scores = _sharded(q, x, k, [shard_bounds(n, world, r) for r in range(world)], pairs=True)
    torch.cuda.synchronize()
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i.cpu().numpy(), ref_s.cpu().numpy())


def test_shared_seed_uneven_shards_with_unsampled_one():
    # one shard too small to sample (its sample is all -inf) and one empty shard
    b, n, k = 256, 300_000, 64
    q = make_int_rows(b, 128, seed=21, device="cuda")
    x = make_int_rows(n, 128, seed=22, device="cuda")
    bounds = [(0, 3_001), (3_001, 3_001), (3_001, 170_000), (170_000, n)]
    ref_i, ref_s = ops.dense_topk(q, x, k)
    ids, scores = _sharded(q, x, k, bounds, pairs=True)
    torch.cuda.synchronize()
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i.cpu().numpy(), ref_s.cpu().numpy())


def test_seed_sample_values_are_tile_maxima_bounds():
    # every sampled value is the max of some 128-item tile of the shard, so at
    # least k distinct items score >= the k-th largest sample value
    b, n, k = 200, 500_000, 50
    q = make_int_rows(b, 128, seed=31, device="cuda")
    x = make_int_rows(n, 128, seed=32, device="cuda")
    vals = ops.dense_seed_sample(q, x, k, n)
    _, ref_s = ops.dense_topk(q, x, k)
    kth_sample = vals.sort(dim=1, descending=True).values[:, k - 1]
    assert bool((kth_sample <= ref_s[:, k - 1]).all())
    assert bool(torch.isfinite(vals).all())


def test_graphed_search_matches_plain_search_on_new_queries():
    from retrieve_b200.shard import GraphedSearch, ShardedDenseTopK

    b, n, k = 512, 300_000, 100
    x = make_int_rows(n, 128, seed=41, device="cuda")
    index = ShardedDenseTopK(x, 0, k)
    q0 = make_int_rows(b, 128, seed=42, device="cuda")
    g = GraphedSearch(index, q0)
    for seed in (43, 44):
        qn = make_int_rows(b, 128, seed=seed, device="cuda")
        ref_i, ref_s = index.search(qn)
        ids, scores = g.search(qn.cpu().pin_memory())
        torch.cuda.synchronize()
        assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_i.cpu().numpy(), ref_s.cpu().numpy())
    g.release()
