"""The IVF build's k-means restated on the CPU (retrieve/src/retrieve/indexing/kmeans.py:15-122).
Test infrastructure: only the tests use it, as the checker.

Lloyd's algorithm under inner product: assignment = argmax of ``x . c`` (first index on ties;
fp32 products summed by numpy), centroid = the cluster's mean from fp64 sums added in row order
and rounded to fp32, divided in fp32 by the count (an empty cluster keeps its centroid); seeds
from ``n_lists`` distinct rows (``torch.randperm`` on a CPU generator seeded with ``seed``) or
k-means++ D^2 sampling with the reference's draws: the first row ``torch.randint``, then for
each next seed a ``torch.rand`` times the cumsum's total, located by a right-sided search of the
cumsum of ``max(0, |x|^2 - 2 x.c + |c|^2)`` (clamped to the last row). ``torch`` is used only for
the seeded draws, so the draw sequence is the reference's.
"""

from __future__ import annotations

import numpy as np
import torch


def assign(x, centroids):
    """Row -> the centroid of largest inner product, first index on ties."""
    return (np.asarray(x, np.float32) @ np.asarray(centroids, np.float32).T).argmax(axis=1).astype(np.int64)


def cluster_sums(x, assignments, n_lists):
    """fp64 sums of each cluster's rows, added in row order, and the counts; rows assigned
    outside ``[0, n_lists)`` are left out."""
    x = np.asarray(x, dtype=np.float64)
    a = np.asarray(assignments, dtype=np.int64)
    keep = (a >= 0) & (a < n_lists)
    sums = np.zeros((n_lists, x.shape[1]), dtype=np.float64)
    np.add.at(sums, a[keep], x[keep])  # unbuffered, in row order
    return sums, np.bincount(a[keep], minlength=n_lists).astype(np.int64)


def _seed_kmeanspp(x, n_lists, gen):
    n = x.shape[0]
    sq = (x * x).sum(axis=1, dtype=np.float32)
    seeds = np.empty((n_lists, x.shape[1]), dtype=np.float32)
    seeds[0] = x[int(torch.randint(n, (1,), generator=gen)[0])]

    def dist(c):
        return np.maximum(sq - np.float32(2) * (x @ c) + np.dot(c, c), np.float32(0)).astype(np.float32)

    d2 = dist(seeds[0])
    for j in range(1, n_lists):
        cdf = np.cumsum(d2, dtype=np.float32)
        draw = np.float32(float(torch.rand((), generator=gen))) * cdf[-1]
        row = min(int(np.searchsorted(cdf, draw, side="right")), n - 1)
        seeds[j] = x[row]
        d2 = np.minimum(d2, dist(x[row]))
    return seeds


def fit(x, n_lists, n_iter=10, seed=0, init="random"):
    """``KMeans(n_lists, n_iter, seed, init).fit(x)``: ``(centroids fp32, assignments int64)``."""
    x = np.asarray(x, dtype=np.float32)
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    if init == "kmeans++":
        centroids = _seed_kmeanspp(x, n_lists, gen)
    else:
        centroids = x[torch.randperm(x.shape[0], generator=gen)[:n_lists].numpy()].copy()
    for _ in range(n_iter):
        sums, counts = cluster_sums(x, assign(x, centroids), n_lists)
        cnt = counts.astype(np.float32)
        means = sums.astype(np.float32) / np.maximum(cnt, np.float32(1))[:, None]
        centroids = np.where((cnt > 0)[:, None], means, centroids).astype(np.float32)
    return centroids, assign(x, centroids)
