"""Regenerates ``tests/golden/golden_kmeans.npz``: the REFERENCE's ``KMeans``
(retrieve/src/retrieve/indexing/kmeans.py:15-122) run on the CPU by its own code:

    PYTHONPATH=<reference>/retrieve/src python tests/golden/make_golden_kmeans.py

The data is chosen so that every sum the algorithm forms is exact in the arithmetic it uses,
and the result depends on the algorithm and its draws only, not on the reduction order of a
device or library: 500 rows of D = 16 values ``k / 16`` (|k| <= 16) around 8 well-separated
centres. Squared distances are multiples of 1/256 below 2^8, so their fp32 cumsum over 500 rows
is exact; the cluster sums are exact in fp64; the assignment margins are wide.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
N, D, N_LISTS, N_ITER = 500, 16, 8, 5


def data() -> np.ndarray:
    g = torch.Generator().manual_seed(5)
    centres = torch.randint(-10, 11, (N_LISTS, D), generator=g)
    which = torch.randint(0, N_LISTS, (N,), generator=g)
    noise = torch.randint(-3, 4, (N, D), generator=g)
    return ((centres[which] + noise).clamp(-16, 16).float() / 16).numpy()


def main() -> None:
    from retrieve.indexing.kmeans import KMeans

    x = data()
    out = {"x": x}
    for init in ("random", "kmeans++"):
        for seed in (0, 3):
            c, a = KMeans(N_LISTS, N_ITER, seed=seed, init=init).fit(torch.from_numpy(x))
            key = f"{init.replace('+', 'p')}_{seed}"
            out[key + "_centroids"] = c.numpy()
            out[key + "_assign"] = a.numpy()
    np.savez_compressed(HERE / "golden_kmeans.npz", **out)
    print("wrote", HERE / "golden_kmeans.npz", sorted(out))


if __name__ == "__main__":
    main()
