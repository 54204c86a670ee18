"""SilverTorch's expression parser (``st::parse_expression_query_batch``) served by the
library's host parser (retrieve_b200/csrc/st_parser.cpp), against the reference's own CPU
parser: tests/golden/golden_parser.npz (made by tests/golden/make_golden_parser.py) and the
plans of tests/golden/golden_bloom_st.npz. CPU only."""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from retrieve_b200 import _lib

HERE = Path(__file__).resolve().parent
GOLDEN = np.load(HERE / "golden" / "golden_parser.npz")
META = json.loads(str(GOLDEN["meta"]))
BLOOM = np.load(HERE / "golden" / "golden_bloom_st.npz")

PINNED = (  # retrieve/tests/parity/test_official.py:87-90
    "st::parse_expression_query_batch(str[] expressions, Tensor silvertorch_ks, "
    "int bloom_hash_k, bool return_query_plan=True, int max_sub_queries=5) -> (int, Tensor[])"
)


def _parse(exprs, hash_k=7, return_plan=True, max_sub=5):
    import retrieve_b200.st  # noqa: F401  (registers the ops)

    return torch.ops.st.parse_expression_query_batch(exprs, torch.ones(len(exprs), dtype=torch.int64), hash_k,
                                                     return_plan, max_sub)


def test_schema_is_the_reference_one():
    _parse([])
    assert str(torch.ops.st.parse_expression_query_batch.default._schema) == PINNED


@pytest.mark.parametrize("ci", range(len(META["cases"])))
def test_plans_are_byte_identical(ci):
    case = META["cases"][ci]
    stack, (data, offsets) = _parse(case["expressions"], case["hash_k"], True, case["max_sub_queries"])
    assert data.dtype == torch.int8 and offsets.dtype == torch.int64
    assert stack == int(GOLDEN[f"c{ci}_stack"])
    assert np.array_equal(offsets.numpy(), GOLDEN[f"c{ci}_offsets"])
    assert np.array_equal(data.numpy(), GOLDEN[f"c{ci}_data"])
    stack2, (d2, o2) = _parse(case["expressions"], case["hash_k"], False, case["max_sub_queries"])
    assert stack2 == stack and d2.numel() == 0 and o2.numel() == 0


def test_bloom_fixture_plans_are_reproduced():
    from tests.golden.make_golden_bloom_st import EXPRESSIONS, HASH_K

    stack, (data, offsets) = _parse(EXPRESSIONS, HASH_K)
    assert stack == int(BLOOM["max_stack"])
    assert np.array_equal(data.numpy(), BLOOM["plan_data"]) and np.array_equal(offsets.numpy(), BLOOM["plan_offsets"])


@pytest.mark.parametrize("expr", META["rejected"])
def test_malformed_expressions_raise(expr):
    with pytest.raises(RuntimeError, match="parse_expression_query_batch"):
        _parse(["1:1", expr])


def test_deep_nesting_raises_instead_of_overflowing():
    for expr in ("(" * 6000 + "1:2" + ")" * 6000, "!" * 9000 + "1:2"):
        with pytest.raises(RuntimeError, match="nested too deeply"):
            _parse([expr])
    stack, _ = _parse(["(" * 300 + "1:2" + ")" * 300, "!" * 900 + "1:2"])
    assert stack == 1


def test_capi_size_query_and_buffers():
    lib = _lib.lib()
    exprs = [b"1:2 AND 3:4", b""]
    bufs = (ctypes.c_char_p * 2)(*exprs)
    lens = (ctypes.c_int64 * 2)(*[len(e) for e in exprs])
    nbytes, stack = ctypes.c_int64(0), ctypes.c_int64(0)
    assert lib.rb_st_parse_expression_batch(bufs, lens, 2, 7, 5, None, 0, None, ctypes.byref(nbytes),
                                            ctypes.byref(stack)) == _lib.RB_OK
    assert stack.value == 2 and nbytes.value > 0
    small = (ctypes.c_int8 * 8)()
    offs = (ctypes.c_int64 * 16)()
    assert lib.rb_st_parse_expression_batch(bufs, lens, 2, 7, 5, small, 8, offs, ctypes.byref(nbytes),
                                            ctypes.byref(stack)) == _lib.RB_ERR_WORKSPACE
    assert lib.rb_st_parse_expression_batch(bufs, lens, 2, 0, 5, None, 0, None, ctypes.byref(nbytes),
                                            ctypes.byref(stack)) == _lib.RB_ERR_INVALID_ARG  # hash_k < 1
    bad = (ctypes.c_char_p * 1)(b"1:2 )")
    assert lib.rb_st_parse_expression_batch(bad, (ctypes.c_int64 * 1)(5), 1, 7, 5, None, 0, None,
                                            ctypes.byref(nbytes), ctypes.byref(stack)) == _lib.RB_ERR_INVALID_ARG
    assert b"position 4" in lib.rb_last_error()


def test_plans_drive_the_bloom_oracle():
    """Plans from this parser, run by the bloom restatement over the reference's index, give
    the reference's bloom masks (the plans are the reference's bytes, so this closes the loop)."""
    from oracle import ivf
    from tests.golden.make_golden_bloom_st import EXPRESSIONS, HASH_K

    _, (data, offsets) = _parse(EXPRESSIONS, HASH_K)
    n = int(BLOOM["n"])
    want = np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n].astype(bool)
    for p in (0, 4, 5, 9):
        got = ivf.bloom_plan_mask(BLOOM["bloom_index"], BLOOM["bundle_b_offsets"], data.numpy(), offsets.numpy(), p,
                                  int(BLOOM["k"]), HASH_K, n)
        assert np.array_equal(got, want[p])
