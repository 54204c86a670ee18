"""Failure paths without a GPU fault: the bounded waits of the pipelined kernels run out
on a barrier that nothing completes, write their timeout code where the host reads it, and
leave the context usable (rb_wait_probe, through the scan kernels' own bounded wait with a
short limit). The host-side failure of a rank between steps is in test_shard_gloo.py."""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from retrieve_b200 import _lib


def test_wait_probe_checks_its_arguments_without_a_device():
    lib = _lib.lib()
    fake = ctypes.c_void_p(256)
    assert lib.rb_wait_probe(10, fake, 4096, None) == _lib.RB_ERR_INVALID_ARG  # below 1 us
    assert lib.rb_wait_probe(3_000_000_000, fake, 4096, None) == _lib.RB_ERR_INVALID_ARG  # above 2 s
    assert lib.rb_wait_probe(1_000_000, None, 4096, None) == _lib.RB_ERR_INVALID_ARG
    assert lib.rb_wait_probe(1_000_000, fake, 128, None) == _lib.RB_ERR_INVALID_ARG


@pytest.mark.gpu
@pytest.mark.parametrize("limit_ms", [20, 200])
def test_bounded_wait_runs_out_and_reports(limit_ms):
    lib = _lib.lib()
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(lib.rb_wait_probe(limit_ms * 1_000_000, ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
               "wait_probe")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    err = ctypes.c_int(0)
    _lib.check(lib.rb_workspace_device_error(ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.byref(err)), "err")
    assert err.value in (1, 2, 3)  # a role's timeout code
    assert limit_ms / 1e3 <= elapsed < limit_ms / 1e3 + 2.0
    # the context is still usable: a search right after gives the exact answer
    from oracle.dense import dense_topk as oracle_dense_topk
    from retrieve_b200 import ops

    g = torch.Generator().manual_seed(3)
    q = torch.randint(-3, 4, (8, 128), generator=g).to(torch.bfloat16)
    x = torch.randint(-3, 4, (3000, 128), generator=g).to(torch.bfloat16)
    ids, scores = ops.dense_topk(q.cuda(), x.cuda(), 10)
    ref_i, ref_s = oracle_dense_topk(q, x, 10)
    assert np.array_equal(scores.cpu().numpy(), ref_s) and np.array_equal(ids.cpu().numpy(), ref_i)
