"""CPU checks of the C-ABI boundary: the library builds, loads without a GPU and
exports every entry point the public header declares; argument errors map to
the reference's exception types without touching a device."""

from __future__ import annotations

import ctypes

import pytest

from retrieve_b200 import _lib


def test_library_exports_every_header_symbol():
    lib = _lib.lib()
    names = _lib.header_symbols()
    assert len(names) >= 5
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    assert set(_lib._SIGNATURES) >= set(names), "ctypes signatures missing for some header symbols"


def test_abi_version():
    assert _lib.lib().rb_abi_version() == 1


def test_dense_workspace_query_is_host_only():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.rb_dense_topk_workspace_size(1024, 10_000_000, 128, _lib.RB_BF16, 100, ctypes.byref(n)) == 0
    assert 10 << 20 < n.value < 1 << 30
    assert lib.rb_dense_topk_workspace_size(4, 10, 128, _lib.RB_BF16, 0, ctypes.byref(n)) == _lib.RB_ERR_INVALID_ARG
    assert b"k" in lib.rb_last_error()


def test_dense_argument_errors_map_to_python_exceptions():
    lib = _lib.lib()
    rc = lib.rb_dense_topk(None, None, 4, 10, 128, 7, 10, 0, None, None, None, 0, None)
    with pytest.raises(TypeError):
        _lib.check(rc, "dense_topk")
    rc = lib.rb_dense_topk(None, None, 4, 10, 96, _lib.RB_BF16, 10, 0, None, None, None, 0, None)
    with pytest.raises(ValueError):
        _lib.check(rc, "dense_topk")
