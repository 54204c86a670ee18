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
    assert _lib.lib().rb_abi_version() == 2


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


def test_workspace_grows_with_row_width_and_k():
    lib = _lib.lib()
    sizes = {}
    for name, d, dt, k in [("bf16 d128", 128, _lib.RB_BF16, 100), ("bf16 d256", 256, _lib.RB_BF16, 100),
                           ("int8 d512", 512, _lib.RB_I8, 100), ("e4m3 d512", 512, _lib.RB_E4M3, 1000),
                           ("bf16 k1024", 128, _lib.RB_BF16, 1024)]:
        n = ctypes.c_size_t(0)
        assert lib.rb_dense_topk_workspace_size(1024, 1_000_000, d, dt, k, ctypes.byref(n)) == 0, name
        sizes[name] = n.value
    # one query group per CTA pair (512-byte rows, lists past 512 entries) halves the
    # splits and doubles the lists per split: k = 1000 needs the largest lists
    assert sizes["e4m3 d512"] > sizes["bf16 d128"]
    assert sizes["bf16 k1024"] > sizes["bf16 d128"]


def test_new_entry_points_validate_before_touching_a_device():
    lib = _lib.lib()
    # e4m3 scan takes no scales
    rc = lib.rb_dense_topk_scaled(None, ctypes.c_void_p(16), None, None, 4, 10, 128, _lib.RB_E4M3, 10, 0, None,
                                  None, None, 0, None)
    assert rc == _lib.RB_ERR_UNSUPPORTED and b"scales" in lib.rb_last_error()
    # only e4m3 rows
    rc = lib.rb_dense_topk_scaled(None, None, None, None, 4, 10, 128, _lib.RB_BF16, 10, 0, None, None, None, 0,
                                  None)
    with pytest.raises(TypeError):
        _lib.check(rc, "dense_topk_scaled")
    # k beyond the selection limit
    rc = lib.rb_dense_topk(None, None, 4, 10, 128, _lib.RB_BF16, 2000, 0, None, None, None, 0, None)
    assert rc == _lib.RB_ERR_UNSUPPORTED and b"1024" in lib.rb_last_error()
    # 1-bit expansion: sizes and alignment
    assert lib.rb_bits_to_pm1(None, -1, 8, None, None) == _lib.RB_ERR_INVALID_ARG
    assert lib.rb_bits_to_pm1_e4m3(ctypes.c_void_p(16), 4, 8, ctypes.c_void_p(17), None) == _lib.RB_ERR_INVALID_ARG
    assert b"aligned" in lib.rb_last_error()
    # sample width of the shared seed
    rc = lib.rb_dense_seed_sample(None, None, 4, 10, 128, _lib.RB_BF16, 10, 11, 10, ctypes.c_void_p(16), None, 0,
                                  None)
    assert rc in (_lib.RB_ERR_INVALID_ARG, _lib.RB_ERR_WORKSPACE)
    rc = lib.rb_dense_topk_seeded(None, None, 4, 10, 128, _lib.RB_BF16, 10, 0, 10, ctypes.c_void_p(16), 2, 11,
                                  None, None, None, None, 0, None)
    assert rc == _lib.RB_ERR_INVALID_ARG and b"m <= k" in lib.rb_last_error()
    # merge of packed pairs
    assert lib.rb_merge_pairs(None, 0, 4, 10, 10, None, None, None) == _lib.RB_ERR_INVALID_ARG
    assert lib.rb_merge_pairs(None, 2, 4, 10, 2000, None, None, None) == _lib.RB_ERR_UNSUPPORTED


def test_noalloc_checks_arguments_like_the_workspace_entry_point():
    """The entry point without a workspace answers a bad call with rb_dense_topk's code,
    even when that call would also need more than its static scratch."""
    lib = _lib.lib()
    big = (4096, 10_000_000)
    for dtype, d, k, want in ((_lib.RB_I8, 128, 100, _lib.RB_ERR_TYPE), (_lib.RB_E4M3, 128, 100, _lib.RB_ERR_TYPE),
                              (_lib.RB_BF16, 128, 2000, _lib.RB_ERR_UNSUPPORTED),
                              (_lib.RB_BF16, 96, 100, _lib.RB_ERR_UNSUPPORTED),
                              (_lib.RB_BF16, 128, 0, _lib.RB_ERR_INVALID_ARG)):
        ref = lib.rb_dense_topk(None, None, *big, d, dtype, k, 0, None, None, None, 0, None)
        got = lib.rb_dense_topk_noalloc(None, None, *big, d, dtype, k, 0, None, None, None)
        assert ref == got == want, (dtype, d, k)
    rc = lib.rb_dense_topk_noalloc(None, None, *big, 128, _lib.RB_BF16, 100, 0, None, None, None)
    assert rc == _lib.RB_ERR_WORKSPACE and b"static" in lib.rb_last_error()


def test_filter_struct_layout_matches_the_header(tmp_path):
    """The ctypes twin of rb_st_filter has the C compiler's field offsets and size (a
    mismatch would hand the kernels shifted pointers)."""
    import shutil
    import subprocess
    from pathlib import Path

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    names = [name for name, _ in _lib.StFilter._fields_]
    src = tmp_path / "layout.c"
    src.write_text(
        "#include <stdio.h>\n#include <stddef.h>\n#include \"retrieve_b200.h\"\nint main(void) {\n"
        + "".join(f'  printf("{n} %zu\\n", offsetof(rb_st_filter, {n}));\n' for n in names)
        + '  printf("size %zu\\n", sizeof(rb_st_filter));\n  return 0;\n}\n'
    )
    exe = tmp_path / "layout"
    include = Path(__file__).resolve().parent.parent / "include"
    subprocess.run([cc, "-I", str(include), str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                         text=True).stdout.splitlines())
    for n in names:
        assert int(got[n]) == getattr(_lib.StFilter, n).offset, n
    assert int(got["size"]) == ctypes.sizeof(_lib.StFilter)
