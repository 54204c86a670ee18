"""The all-gather through the peers' memory (rb_peer_allgather, shard.PeerExchange): one
process per GPU (2 to 4 GPUs; skipped with fewer), host handles over gloo. Every rank
checks the stacks of several steps (the two buffer parities reused), a block that needs
padding to 16 bytes, replays of a captured graph, and a row-sharded dense search through
it, bit for bit the single-GPU search. The CPU test checks the C-ABI's argument errors."""

from __future__ import annotations

import ctypes
import os

import pytest
import torch

from retrieve_b200 import _lib


def test_peer_allgather_checks_its_arguments_without_a_device():
    lib = _lib.lib()
    fake = ctypes.c_void_p(256)
    bases = (ctypes.c_void_p * 2)(256, 512)
    call = lambda **kw: lib.rb_peer_allgather(  # noqa: E731
        kw.get("bases", bases), kw.get("W", 2), kw.get("rank", 0), kw.get("slot", 1024), kw.get("src", fake),
        kw.get("nbytes", 512), fake, fake, fake, kw.get("out", fake), None)
    assert call(W=0) == _lib.RB_ERR_INVALID_ARG
    assert call(rank=2) == _lib.RB_ERR_INVALID_ARG
    assert call(nbytes=2048) == _lib.RB_ERR_INVALID_ARG  # larger than a slot
    assert call(nbytes=20) == _lib.RB_ERR_INVALID_ARG  # not a multiple of 16
    assert call(src=ctypes.c_void_p(264)) == _lib.RB_ERR_INVALID_ARG  # unaligned source
    assert lib.rb_peer_buffer_bytes(4, 1024) == 4 * 64 + 8 * 1024


def _rank(rank, world, port, failures):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta

        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from retrieve_b200 import ops
        from retrieve_b200.shard import PeerExchange, ShardedDenseTopK, shard_bounds

        ex = PeerExchange(4096, dev)
        for step in range(5):  # both parities, several times
            t = torch.full((256,), rank * 100 + step, dtype=torch.int32, device=dev)
            out = ex.allgather(t)
            want = torch.stack([torch.full((256,), r * 100 + step, dtype=torch.int32, device=dev)
                                for r in range(world)])
            assert torch.equal(out, want), f"step {step}"
        t = torch.arange(5, dtype=torch.int32, device=dev) + 10 * rank  # 20 bytes: padded to 32
        out = ex.allgather(t)
        assert torch.equal(out, torch.stack([torch.arange(5, dtype=torch.int32, device=dev) + 10 * r
                                             for r in range(world)]))
        # a captured graph replays the exchange (the step counter is on the device)
        static = torch.zeros(64, dtype=torch.float32, device=dev)
        ex.allgather(static)
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gout = ex.allgather(static)
        for rep in range(3):
            static.fill_(rank + 0.5 * rep)
            graph.replay()
            torch.cuda.synchronize()
            want = torch.stack([torch.full((64,), r + 0.5 * rep, device=dev) for r in range(world)])
            assert torch.equal(gout, want), f"replay {rep}"
        dist.barrier()
        del graph
        assert ex.device_error() == 0
        ex.close()

        # the row-sharded dense search through the peers' memory equals one GPU's
        g = torch.Generator().manual_seed(3)
        n, b, k = 50_000, 300, 100
        x = torch.randint(-3, 4, (n, 128), generator=g).to(torch.bfloat16).to(dev)
        q = torch.randint(-3, 4, (b, 128), generator=g).to(torch.bfloat16).to(dev)
        lo, hi = shard_bounds(n, world, rank)
        index = ShardedDenseTopK(x[lo:hi].contiguous(), lo, k, n_total=n, exchange="peer")
        for _ in range(3):
            ids, scores = index.search(q)
        want_i, want_s = ops.dense_topk(q, x, k)
        assert torch.equal(scores, want_s) and torch.equal(ids, want_i), "sharded search"
        index.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001  (reported to the parent)
        failures[rank] = f"{type(exc).__name__}: {exc}"


@pytest.mark.gpu
def test_peer_allgather_across_gpus():
    n_gpu = torch.cuda.device_count()
    if n_gpu < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp

    world = min(n_gpu, 4)
    mgr = mp.get_context("spawn").Manager()
    failures = mgr.dict()
    mp.start_processes(_rank, args=(world, 29731, failures), nprocs=world, join=True, start_method="spawn")
    assert not dict(failures), dict(failures)
