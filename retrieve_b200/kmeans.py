"""The IVF build's k-means on the device, under the reference's interface
(``retrieve.indexing.kmeans.KMeans``, retrieve/src/retrieve/indexing/kmeans.py:15-122): Lloyd's
algorithm under inner product (a row joins the centroid of largest ``x . c``; a centroid is its
cluster's plain mean; an empty cluster keeps its centroid), seeded from ``n_lists`` distinct
rows or by k-means++ D^2 sampling, every draw from a CPU generator seeded with ``seed``.

What runs where:

* the assignment is a chunked fp32 matmul (cuBLAS) + ``argmax`` (first index on ties), as the
  reference's, so that the IVF lists are the reference's;
* the centroid update is ``rb_kmeans_cluster_sums`` (csrc/kmeans.cu): a stable counting sort of
  the rows by cluster and fp64 sums in row order, ``N x D`` additions where the reference's
  one-hot fp64 GEMMs spend ``n_lists x N x D`` multiply-adds; bit-for-bit reproducible run to
  run, and equal to the reference's sums whenever the fp64 additions are exact;
* k-means++ seeding draws exactly as the reference does (first row uniform; then a CPU uniform
  times the device cumsum of the squared distances, located by ``searchsorted`` with
  ``right=True``), so both give the same seeds on the same device.

CUDA tensors only: the update has no CPU path.
"""

from __future__ import annotations

import ctypes
from typing import Literal

import torch
from torch import Tensor

from retrieve_b200 import _lib

KMeansInit = Literal["random", "kmeans++"]

_DTYPE = {torch.float32: _lib.RB_F32, torch.float16: _lib.RB_F16, torch.bfloat16: _lib.RB_BF16}


def _rows_per_chunk(n: int) -> int:
    return max(1, min(n, 1 << 14))


def cluster_sums(embs: Tensor, assignments: Tensor, n_lists: int) -> tuple[Tensor, Tensor]:
    """``(sums fp64 [n_lists, D], counts int64 [n_lists])`` of ``embs`` [N, D] (fp32 / fp16 /
    bf16, CUDA) grouped by ``assignments`` [N]; rows assigned outside ``[0, n_lists)`` are left
    out."""
    if not embs.is_cuda:
        raise ValueError("cluster_sums runs on CUDA tensors only")
    if embs.dim() != 2 or assignments.dim() != 1 or assignments.shape[0] != embs.shape[0]:
        raise ValueError("embs must be [N, D] and assignments [N]")
    if embs.dtype not in _DTYPE:
        raise TypeError(f"embs must be fp32, fp16 or bf16, got {embs.dtype}")
    x = embs.contiguous()
    a = assignments.to(device=x.device, dtype=torch.int64).contiguous()
    n, d = x.shape
    lib = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    rc = lib.rb_kmeans_cluster_sums_workspace_size(n, int(n_lists), ctypes.byref(nbytes))
    if rc != _lib.RB_OK:
        raise ValueError(lib.rb_last_error().decode(errors="replace"))
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=x.device)
    sums = torch.empty((int(n_lists), d), dtype=torch.float64, device=x.device)
    counts = torch.empty(int(n_lists), dtype=torch.int64, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    rc = lib.rb_kmeans_cluster_sums(ctypes.c_void_p(x.data_ptr()), _DTYPE[x.dtype], n, d,
                                    ctypes.c_void_p(a.data_ptr()), int(n_lists), ctypes.c_void_p(sums.data_ptr()),
                                    ctypes.c_void_p(counts.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                    stream)
    if rc != _lib.RB_OK:
        raise RuntimeError(f"kmeans cluster_sums: {lib.rb_last_error().decode(errors='replace')} (status {rc})")
    return sums, counts


class KMeans:
    """``KMeans(n_lists, n_iter=10, seed=0, init="random")``; ``fit(embs)`` returns
    ``(centroids fp32 [n_lists, D], assignments int64 [N])``, the reference's results (see the
    module docstring for the one difference in arithmetic)."""

    def __init__(self, n_lists: int, n_iter: int = 10, seed: int = 0, init: KMeansInit = "random") -> None:
        if init not in ("random", "kmeans++"):
            raise ValueError(f"init must be 'random' or 'kmeans++', got {init!r}")
        self.n_lists = n_lists
        self.n_iter = n_iter
        self.seed = seed
        self.init = init

    def fit(self, embs: Tensor) -> tuple[Tensor, Tensor]:
        if not embs.is_cuda:
            raise ValueError("KMeans.fit runs on CUDA tensors only")
        n = embs.shape[0]
        gen = torch.Generator(device="cpu")
        gen.manual_seed(self.seed)
        if self.init == "kmeans++":
            centroids = self._kmeanspp(embs, gen)
        else:
            centroids = embs[torch.randperm(n, generator=gen)[: self.n_lists]].clone().float()
        for _ in range(self.n_iter):
            sums, counts = cluster_sums(embs, self.assign(embs, centroids), self.n_lists)
            counts = counts.to(torch.float32)
            means = sums.float() / counts.clamp(min=1).unsqueeze(1)
            centroids = torch.where((counts > 0).unsqueeze(1), means, centroids)
        return centroids, self.assign(embs, centroids)

    def _kmeanspp(self, embs: Tensor, gen: torch.Generator) -> Tensor:
        """D^2 seeding: one row uniform, then each next row with probability proportional to its
        squared distance to the nearest seed so far (``|x|^2 - 2 x.c + |c|^2``, clamped at 0)."""
        x = embs.float()
        n = x.shape[0]
        sq = (x * x).sum(dim=1)
        seeds = torch.empty(self.n_lists, x.shape[1], dtype=torch.float32, device=x.device)
        seeds[0] = x[torch.randint(n, (1,), generator=gen)[0]]
        dist = (sq - 2 * torch.mv(x, seeds[0]) + seeds[0].dot(seeds[0])).clamp_min(0)
        for j in range(1, self.n_lists):
            cdf = torch.cumsum(dist, dim=0)
            draw = torch.rand((), generator=gen) * cdf[-1:]
            row = torch.searchsorted(cdf, draw, right=True).clamp_max(n - 1)[0]
            seeds[j] = x[row]
            dist = torch.minimum(dist, (sq - 2 * torch.mv(x, x[row]) + x[row].dot(x[row])).clamp_min(0))
        return seeds

    @staticmethod
    def assign(embs: Tensor, centroids: Tensor) -> Tensor:
        """The centroid of largest inner product per row, int64 [N] (first index on ties)."""
        n = embs.shape[0]
        step = _rows_per_chunk(n)
        out = torch.empty(n, dtype=torch.int64, device=embs.device)
        for lo in range(0, n, step):
            hi = min(lo + step, n)
            out[lo:hi] = (embs[lo:hi].float() @ centroids.t()).argmax(dim=1)
        return out
