"""rb_dense_topk_noalloc: the dense top-k entry point that allocates nothing.

Callers that cannot allocate device memory on the call path (a host whose
device memory is reserved once at start-up by another allocator, or a binding
with no caching allocator, where a cudaMalloc per call would synchronise the
device) get their scratch from one static device array.
This file checks, through the C-ABI, that two calls in a row return exactly what
rb_dense_topk returns with a caller workspace (integer-valued inputs make every
score exact, so the comparison is bit for bit), and that a call needing more
scratch than the array holds is refused with a clear error. It sits last in
collection order so that a failure here leaves every other test already run,
and it works in a fresh process as well as after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from retrieve_b200 import _lib

pytestmark = pytest.mark.gpu


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _int_rows(n, d, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-3, 4, (n, d), generator=g).to(torch.bfloat16).cuda()


def test_noalloc_matches_workspace_entry_point_twice():
    lib = _lib.lib()
    b, n, d, k = 64, 20_000, 128, 50
    q, x = _int_rows(b, d, 101), _int_rows(n, d, 102)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_workspace_size(b, n, d, _lib.RB_BF16, k, ctypes.byref(nb)), "ws")
    assert nb.value <= lib.rb_dense_topk_noalloc_scratch_bytes()
    ws = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
    ref_i = torch.empty(b, k, dtype=torch.int64, device="cuda")
    ref_s = torch.empty(b, k, dtype=torch.float32, device="cuda")
    rc = lib.rb_dense_topk(_vp(q), _vp(x), b, n, d, _lib.RB_BF16, k, 0, _vp(ref_i), _vp(ref_s), _vp(ws),
                           ws.numel(), stream)
    _lib.check(rc, "dense_topk")

    for call in range(2):
        out_i = torch.full((b, k), 7, dtype=torch.int64, device="cuda")
        out_s = torch.full((b, k), 7.0, dtype=torch.float32, device="cuda")
        rc = lib.rb_dense_topk_noalloc(_vp(q), _vp(x), b, n, d, _lib.RB_BF16, k, 0, _vp(out_i), _vp(out_s), stream)
        _lib.check(rc, f"dense_topk_noalloc call {call}")
        torch.cuda.synchronize()
        assert np.array_equal(out_s.cpu().numpy(), ref_s.cpu().numpy()), f"scores differ on call {call}"
        assert np.array_equal(out_i.cpu().numpy(), ref_i.cpu().numpy()), f"ids differ on call {call}"


def test_noalloc_refuses_more_than_its_static_scratch():
    lib = _lib.lib()
    b, n, d, k = 4096, 10_000_000, 128, 100
    nb = ctypes.c_size_t(0)
    _lib.check(lib.rb_dense_topk_workspace_size(b, n, d, _lib.RB_BF16, k, ctypes.byref(nb)), "ws")
    assert nb.value > lib.rb_dense_topk_noalloc_scratch_bytes()
    rc = lib.rb_dense_topk_noalloc(None, None, b, n, d, _lib.RB_BF16, k, 0, None, None, None)
    assert rc == _lib.RB_ERR_WORKSPACE
    assert b"static" in lib.rb_last_error()
