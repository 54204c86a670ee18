"""Regenerates ``tests/golden/golden_int8.npz`` with the REFERENCE's own
SilverTorch CPU op ``st.fused_kmean_ann`` (built from the read-only checkout by
``oracle/build_ref.py`` into ``oracle/_ref/``):

    python oracle/build_ref.py <reference checkout>
    python tests/golden/make_golden_int8.py

One cluster holding every item, every query probing it, ``divisor_for_int8 =
-1``: the op returns the raw int32 dot of every (query, item) pair
(silvertorch fused_kmean_ann.cpp:60-70, 186-214) — SilverTorch's int8 scoring
with nothing probed away, the raw-dot half of config 4's bit-exact gate. Codes
are uniform int8 (the full [-128, 127] range, so products reach 2^14 and sums
exercise the int32 accumulation at D = 256).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main() -> None:
    lib = HERE.parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"
    torch.ops.load_library(str(lib))
    st = torch.ops.st
    out = {}
    for d, (b, n) in {128: (24, 1000), 256: (16, 777)}.items():
        g = torch.Generator().manual_seed(d)
        items = torch.randint(-128, 128, (n, d), generator=g, dtype=torch.int64).to(torch.int8)
        queries = torch.randint(-128, 128, (b, d), generator=g, dtype=torch.int64).to(torch.int8)
        offsets = torch.tensor([0, n], dtype=torch.int64)
        cluster_ids = torch.zeros((b, 1), dtype=torch.int64)
        cluster_len = torch.full((b, 1), n, dtype=torch.int64)
        scores, idx = st.fused_kmean_ann(offsets, cluster_ids, cluster_len, items, queries, n, None, -1, -1, None,
                                         None)
        assert scores.dtype == torch.int32 and idx[:, :n].eq(torch.arange(n, dtype=torch.int32)).all()
        out[f"items_{d}"] = items.numpy()
        out[f"queries_{d}"] = queries.numpy()
        out[f"dots_{d}"] = scores[:, :n].numpy()
    np.savez_compressed(HERE / "golden_int8.npz", **out)
    print("wrote", HERE / "golden_int8.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
