"""The IVF build's k-means (retrieve_b200/kmeans.py, csrc/kmeans.cu) against the reference's
``KMeans`` run on the CPU (tests/golden/golden_kmeans.npz, made by
tests/golden/make_golden_kmeans.py) and the restatement in oracle/kmeans.py."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kmeans as okm
from retrieve_b200 import _lib

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden_kmeans.npz")
CASES = [("random", 0), ("random", 3), ("kmeans++", 0), ("kmeans++", 3)]


def _key(init, seed):
    return f"{init.replace('+', 'p')}_{seed}"


@pytest.mark.parametrize("init,seed", CASES)
def test_oracle_matches_reference_kmeans(init, seed):
    c, a = okm.fit(GOLDEN["x"], 8, 5, seed=seed, init=init)
    assert np.array_equal(c, GOLDEN[_key(init, seed) + "_centroids"])
    assert np.array_equal(a, GOLDEN[_key(init, seed) + "_assign"])


def test_oracle_cluster_sums_leave_out_unassigned_rows():
    x = np.arange(12, dtype=np.float32).reshape(6, 2)
    sums, counts = okm.cluster_sums(x, np.array([0, 2, -1, 2, 5, 0]), 3)
    assert counts.tolist() == [2, 0, 2]
    assert sums.tolist() == [[10, 12], [0, 0], [8, 10]]


def test_capi_checks_need_no_device():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.rb_kmeans_cluster_sums_workspace_size(10_000_000, 1024, ctypes.byref(n)) == _lib.RB_OK
    assert n.value >= 10_000_000 * 8  # the sorted row order, at least
    assert lib.rb_kmeans_cluster_sums_workspace_size(10, 0, ctypes.byref(n)) == _lib.RB_ERR_INVALID_ARG
    assert lib.rb_kmeans_cluster_sums_workspace_size(10, 1 << 25, ctypes.byref(n)) == _lib.RB_ERR_INVALID_ARG
    fake = ctypes.c_void_p(16)  # never dereferenced: the checks fail first
    assert lib.rb_kmeans_cluster_sums(fake, _lib.RB_I8, 10, 4, fake, 3, fake, fake, None, 0, None) == _lib.RB_ERR_TYPE
    assert lib.rb_kmeans_cluster_sums(fake, _lib.RB_F32, 10, 4, fake, 3, fake, fake, None, 0,
                                      None) == _lib.RB_ERR_WORKSPACE
    assert lib.rb_kmeans_cluster_sums(fake, _lib.RB_F32, 10, 0, fake, 3, fake, fake, None, 0,
                                      None) == _lib.RB_ERR_INVALID_ARG


def test_cpu_tensors_are_refused():
    from retrieve_b200.kmeans import KMeans, cluster_sums

    with pytest.raises(ValueError, match="CUDA"):
        KMeans(4).fit(torch.zeros(10, 4))
    with pytest.raises(ValueError, match="CUDA"):
        cluster_sums(torch.zeros(10, 4), torch.zeros(10, dtype=torch.int64), 4)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("n,n_lists", [(50_000, 37), (3_000, 1), (120_000, 1000), (0, 5)])
def test_cluster_sums_match_row_order_fp64(dtype, n, n_lists):
    """fp64 sums in row order, bit for bit the restatement's (numpy's unbuffered add in row
    order), counts included; rows assigned outside [0, n_lists) left out; two calls identical."""
    from retrieve_b200.kmeans import cluster_sums

    g = torch.Generator().manual_seed(n + n_lists)
    x = torch.randn(n, 72, generator=g).to(dtype)
    a = torch.randint(-2, n_lists + 2, (n,), generator=g)
    sums, counts = cluster_sums(x.cuda(), a.cuda(), n_lists)
    want_s, want_c = okm.cluster_sums(x.float().numpy(), a.numpy(), n_lists)
    assert np.array_equal(counts.cpu().numpy(), want_c)
    assert np.array_equal(sums.cpu().numpy(), want_s)
    sums2, counts2 = cluster_sums(x.cuda(), a.cuda(), n_lists)
    assert torch.equal(sums, sums2) and torch.equal(counts, counts2)


@pytest.mark.gpu
@pytest.mark.parametrize("init,seed", CASES)
def test_kmeans_matches_reference(init, seed):
    """The device k-means on the fixture's data (every sum exact, wide margins): the reference's
    centroids and assignments, bit for bit."""
    from retrieve_b200.kmeans import KMeans

    c, a = KMeans(8, 5, seed=seed, init=init).fit(torch.from_numpy(GOLDEN["x"]).cuda())
    assert np.array_equal(c.cpu().numpy(), GOLDEN[_key(init, seed) + "_centroids"])
    assert np.array_equal(a.cpu().numpy(), GOLDEN[_key(init, seed) + "_assign"])
