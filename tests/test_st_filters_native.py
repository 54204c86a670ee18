"""The per-position filter code of st::search's scan kernels
(retrieve_b200/csrc/st_filters.cuh, host and device) run on the CPU: built with nvcc from
tests/native/st_filters_host.cu and checked against the reference's bloom masks
(tests/golden/golden_bloom_st.npz), the clause predicate pinned to the reference, and the
high-bit-first mask order. No GPU needed."""

from __future__ import annotations

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import filters, ivf

ROOT = Path(__file__).resolve().parent.parent
BLOOM = np.load(Path(__file__).resolve().parent / "golden" / "golden_bloom_st.npz")


@pytest.fixture(scope="module")
def host(tmp_path_factory):
    nvcc = shutil.which("nvcc") or ("/usr/local/cuda/bin/nvcc" if Path("/usr/local/cuda/bin/nvcc").exists() else None)
    if nvcc is None:
        pytest.skip("nvcc is not available")
    out = tmp_path_factory.mktemp("native") / "st_filters_host.so"
    subprocess.run([nvcc, "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-I", str(ROOT / "retrieve_b200" / "csrc"),
                    "-I", str(ROOT / "include"), str(ROOT / "tests" / "native" / "st_filters_host.cu"), "-o", str(out)],
                   check=True)
    return ctypes.CDLL(str(out))


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_bloom_code_reproduces_reference_masks(host):
    n = int(BLOOM["n"])
    want = np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n].astype(bool)
    n_plans = want.shape[0]
    blob = np.ascontiguousarray(ivf.plan_blob(BLOOM["plan_data"], BLOOM["plan_offsets"], n_plans + 2))
    index = np.ascontiguousarray(BLOOM["bloom_index"])
    boff = np.ascontiguousarray(BLOOM["bundle_b_offsets"])
    rows = np.repeat(np.arange(n_plans, dtype=np.int64), n)
    docs = np.tile(np.arange(n, dtype=np.int64), n_plans)
    out = np.zeros(rows.size, dtype=np.uint8)
    f = host.host_bloom_pass
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_int64, ctypes.c_void_p]
    f(_p(index), index.size, _p(boff), boff.size - 1, _p(blob), blob.size, n_plans + 2, None, int(BLOOM["k"]),
      int(BLOOM["hash_k"]), _p(rows), _p(docs), rows.size, _p(out))
    assert np.array_equal(out.reshape(n_plans, n).astype(bool), want)
    # through a plan index (rows -> plans), and a malformed plan slot fails every doc
    plan_index = np.array([3, 3, 0, n_plans + 1], dtype=np.int64)
    rows2 = np.repeat(np.arange(4, dtype=np.int64), n)
    out2 = np.zeros(rows2.size, dtype=np.uint8)
    f(_p(index), index.size, _p(boff), boff.size - 1, _p(blob), blob.size, n_plans + 2, _p(plan_index),
      int(BLOOM["k"]), int(BLOOM["hash_k"]), _p(rows2), _p(np.tile(np.arange(n, dtype=np.int64), 4)), rows2.size,
      _p(out2))
    got = out2.reshape(4, n).astype(bool)
    assert np.array_equal(got[0], want[3]) and np.array_equal(got[2], want[0]) and not got[3].any()


def test_bloom_word_code_reproduces_reference_search(host):
    """bloom_plan_word, the per-column body of the device bloom searches, gives the
    reference's packed st.bloom_index_search_batch words for every plan and column."""
    want = BLOOM["words"]
    n_plans, n_cols = want.shape
    blob = np.ascontiguousarray(ivf.plan_blob(BLOOM["plan_data"], BLOOM["plan_offsets"], n_plans))
    index = np.ascontiguousarray(BLOOM["bloom_index"])
    boff = np.ascontiguousarray(BLOOM["bundle_b_offsets"])
    out = np.zeros((n_plans, n_cols), dtype=np.int64)
    f = host.host_bloom_words
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p]
    f(_p(index), index.size, _p(boff), boff.size - 1, _p(blob), blob.size, n_plans, int(BLOOM["k"]),
      int(BLOOM["hash_k"]), n_plans, n_cols, _p(out))
    assert np.array_equal(out, want)


def test_partial_mask_code_reads_the_reference_partial_response(host):
    """partial_mask_pass over the reference's partial response (one plan a row) keeps doc i of
    probed range (b, j) exactly when the reference's full search passes its sorted position."""
    probe = BLOOM["probe"]
    b, p = probe.shape
    coff, sizes = BLOOM["cluster_offsets"], BLOOM["cluster_sizes"]
    n = int(BLOOM["n"])
    full = np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n].astype(bool)
    rows, probes, docs, want = [], [], [], []
    for r in range(b):
        for j in range(p):
            c = probe[r, j]
            for i in range(int(sizes[c])):
                rows.append(r), probes.append(j), docs.append(i), want.append(full[r, coff[c] + i])
    rows, probes, docs = (np.ascontiguousarray(np.array(x, dtype=np.int64)) for x in (rows, probes, docs))
    out = np.zeros(rows.size, dtype=np.uint8)
    cumsum = np.ascontiguousarray(BLOOM["p_cumsum"])
    first = np.ascontiguousarray(BLOOM["p_first"])
    words = np.ascontiguousarray(BLOOM["p_words"])
    f = host.host_partial_keep
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    f(_p(cumsum), _p(first), _p(words), words.size, p, _p(rows), _p(probes), _p(docs), rows.size, _p(out))
    assert np.array_equal(out.astype(bool), np.array(want))


def test_exact_code_reproduces_clause_predicate(host):
    rng = np.random.default_rng(4)
    n, c = 900, 4
    attrs = rng.integers(-1, 7, (n, c, 3))
    rev = rng.random(c) < 0.5
    q = rng.integers(-1, 7, (12, c))
    q[0, 2] = 2**40
    slots, clause_slots = ivf.exact_layout(attrs)
    qq = np.ascontiguousarray(ivf.exact_query(q))
    slots = np.ascontiguousarray(slots)
    rev8 = np.ascontiguousarray(rev.astype(np.uint8))
    rows = np.repeat(np.arange(q.shape[0], dtype=np.int64), n)
    docs = np.tile(np.arange(n, dtype=np.int64), q.shape[0])
    out = np.zeros(rows.size, dtype=np.uint8)
    f = host.host_exact_pass
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    f(_p(slots), slots.shape[0], slots.shape[1], _p(clause_slots), _p(rev8), _p(qq), c, _p(rows), _p(docs), rows.size,
      _p(out))
    assert np.array_equal(out.reshape(q.shape[0], n).astype(bool), filters.clause_mask(attrs, rev, q))


def test_mask_code_reads_high_bit_first(host):
    rng = np.random.default_rng(6)
    m = rng.random((5, 300)) < 0.5
    words = np.ascontiguousarray(ivf.pack_mask_high_first(m))
    rows = np.repeat(np.arange(5, dtype=np.int64), 300)
    docs = np.tile(np.arange(300, dtype=np.int64), 5)
    out = np.zeros(rows.size, dtype=np.uint8)
    f = host.host_mask_pass
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    f(_p(words), words.shape[1], _p(rows), _p(docs), rows.size, _p(out))
    assert np.array_equal(out.reshape(5, 300).astype(bool), m)


def test_slot_arithmetic_reproduces_the_scorer_layout(host):
    """The grouped scorer's and the sharded finish's slot starts and slot -> position search
    give back every probed position in the reference scorer's slot order (ivf.probe_slots),
    with empty clusters, clusters of whole warps and invalid probe ids (empty)."""
    f = host.host_slot_positions
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    rng = np.random.default_rng(8)
    for _ in range(200):
        n_lists = int(rng.integers(1, 40))
        sizes = rng.integers(0, 130, n_lists).astype(np.int64)
        sizes[rng.random(n_lists) < 0.2] = 64
        offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
        p = int(rng.integers(1, min(n_lists, 12) + 1))
        prow = rng.permutation(n_lists)[:p].astype(np.int64)
        want = ivf.probe_slots(prow, offsets, sizes)
        width = (len(want) + 31) // 32 * 32
        head = np.zeros(p, np.int64)
        tail = np.zeros(p, np.int64)
        got = np.full(max(width, 1), -7, np.int64)
        total = f(_p(prow), p, _p(offsets), _p(sizes), n_lists, int(offsets[-1]), width, _p(head), _p(tail), _p(got))
        assert total == len(want) and np.array_equal(got[: len(want)], want)
    # an invalid probe id scores as an empty cluster
    prow = np.array([0, 99, 1], dtype=np.int64)
    sizes = np.array([40, 33], dtype=np.int64)
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    got = np.full(96, -7, np.int64)
    total = f(_p(prow), 3, _p(offsets), _p(sizes), 2, 73, 96, _p(np.zeros(3, np.int64)), _p(np.zeros(3, np.int64)),
              _p(got))
    assert total == 73 and np.array_equal(got[:73], ivf.probe_slots(np.array([0, 1]), offsets, sizes))


def test_bloom_build_code_reproduces_reference_index(host):
    """The device bloom build's hash, positions, widths and word / bit arithmetic
    (csrc/bloom_hash.cuh) rebuild the reference's CPU-built index bit for bit."""
    fid, off, val = (np.ascontiguousarray(x) for x in ivf.attrs_to_features(BLOOM["attrs"]))
    n, c = BLOOM["attrs"].shape[:2]
    f = host.host_bloom_build
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                  ctypes.c_double, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    boff = np.zeros((n + 2047) // 2048 + 1, np.int64)
    f(_p(fid), _p(off), _p(val), n, c, int(BLOOM["k"]), 10.0, 0, _p(boff), None)
    assert np.array_equal(boff, BLOOM["bundle_b_offsets"])
    index = np.zeros(int(boff[-1]) * 32, np.uint64)
    f(_p(fid), _p(off), _p(val), n, c, int(BLOOM["k"]), 10.0, 0, _p(boff), _p(index))
    assert np.array_equal(index.view(np.int64), BLOOM["bloom_index"])
