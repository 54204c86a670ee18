"""Regenerates ``tests/golden/golden_select.npz``: the REFERENCE's CPU ``st.is_topk``
(silvertorch/ops/csrc/is_topk.cpp:22-80) and ``st.take_top_k_and_gather_from_main_and_fresh``
(fresh_index_post_processing.cpp:226-272), built from the checkout:

    python oracle/build_ref.py <reference checkout>
    python tests/golden/make_golden_select.py

The inputs keep to where the reference's CPU and CUDA ops agree: ``is_topk`` with 1 <= k < n and
no NaN (the CPU op flags nothing for k <= 0, the CUDA op clamps), ``take_top_k`` on untied scores
(``torch.topk`` leaves tie order open), with out-of-range data indices (row 0).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main() -> None:
    torch.ops.load_library(str(HERE.parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"))
    st = torch.ops.st
    g = torch.Generator().manual_seed(11)
    out = {}
    s = torch.randn(6, 50, generator=g)
    s[:, :20] = torch.round(s[:, :20] * 2) / 2  # ties at the k-th value
    ks = torch.randint(1, 50, (6,), generator=g)
    for largest in (True, False):
        flags = torch.zeros(6, 50)
        st.is_topk(s, ks, flags, largest)
        out[f"is_topk_{int(largest)}"] = flags.numpy()
    out["is_topk_scores"], out["is_topk_ks"] = s.numpy(), ks.numpy()

    b, mm, mf = 5, 30, 12
    main_scores = torch.randn(b, mm, generator=g)
    fresh_scores = torch.randn(b, mf, generator=g) + 0.5
    main_idx = torch.randint(-2, 42, (b, mm), generator=g)
    fresh_idx = torch.randint(-1, 22, (b, mf), generator=g)
    main_emb, fresh_emb = torch.randn(40, 4, generator=g), torch.randn(20, 4, generator=g)
    main_id, fresh_id = torch.arange(40) + 1000, torch.arange(20) + 5000
    for k in (7, 60):
        top, cols, fresh, data = st.take_top_k_and_gather_from_main_and_fresh(
            main_scores, fresh_scores, main_idx, fresh_idx, k, ["emb", "id"], [main_emb, main_id],
            [fresh_emb, fresh_id])
        out[f"ttk{k}_top"], out[f"ttk{k}_cols"], out[f"ttk{k}_fresh"] = top.numpy(), cols.numpy(), fresh.numpy()
        out[f"ttk{k}_emb"], out[f"ttk{k}_id"] = data["emb"].numpy(), data["id"].numpy()
    for name, t in (("main_scores", main_scores), ("fresh_scores", fresh_scores), ("main_idx", main_idx),
                    ("fresh_idx", fresh_idx), ("main_emb", main_emb), ("fresh_emb", fresh_emb),
                    ("main_id", main_id), ("fresh_id", fresh_id)):
        out[name] = t.numpy()
    np.savez_compressed(HERE / "golden_select.npz", **out)
    print("wrote", HERE / "golden_select.npz", sorted(out))


if __name__ == "__main__":
    main()
