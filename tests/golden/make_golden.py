"""Regenerates ``tests/golden/golden.npz`` by running the REFERENCE's own torch
path (rmnigm/retrieve, imported from a read-only checkout) on the seeded inputs
of ``golden_inputs.py``:

    PYTHONPATH=<reference>/retrieve/src python tests/golden/make_golden.py

The fixtures pin the CPU oracle (``oracle/``) to the reference's results; the
GPU tests then pin the kernels to the oracle. Nothing at test time imports the
reference.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden import golden_inputs as gi  # noqa: E402


def main() -> None:
    from retrieve.functional import popcount_int64
    from retrieve.indexing.quantize import quantize_int8, quantize_simhash_1bit
    from retrieve.modules.knn import FullScanKNN
    from retrieve.ops import reference as ref

    out: dict[str, np.ndarray] = {}
    torch.set_num_threads(8)

    # config 1: FullScanKNN (knn.py:153-170), fp32 matmul + torch.topk
    q, x = gi.c1_inputs()
    m = FullScanKNN(k=10)
    m.register_index(x)
    ids, scores = m(q)
    out["c1_ids"], out["c1_scores"] = ids.numpy(), scores.numpy()

    # exact clause filter (ops/reference/clause_mask.py, clause_compact.py)
    attrs, rev, qa = gi.clause_inputs()
    out["clause_mask"] = np.packbits(ref.clause_mask(attrs, rev, qa).numpy(), axis=1)
    sc = torch.randn(qa.shape[0], attrs.shape[0], generator=torch.Generator().manual_seed(4))
    out["clause_mask_scores"] = ref.clause_mask_scores(sc, attrs, rev, qa).numpy()
    cids, ccounts = ref.clause_compact(attrs, rev, qa)
    out["clause_counts"] = ccounts.numpy()
    out["clause_ids_head"] = np.stack(
        [np.pad(cids[i, : ccounts[i]].numpy(), (0, attrs.shape[0] - int(ccounts[i])), constant_values=-1)
         for i in range(qa.shape[0])]
    )

    # fused_masked_knn_topk twin (ops/reference/fused_masked_knn_topk.py, CPU fp32 bmm)
    fq, fx, fpos, fcnt = gi.fmkt_inputs()
    fi, fs = ref.fused_masked_knn_topk(fq, fx, fpos, fcnt, 20)
    out["fmkt_ids"], out["fmkt_scores"] = fi.numpy(), fs.numpy()

    # 1-bit twins (ops/reference/oporp_1bit_match_topk.py)
    qb, xb, opos, ocnt = gi.oporp_inputs()
    oi, os_ = ref.oporp_1bit_match_topk_full(qb, xb, 50)
    out["oporp_full_ids"], out["oporp_full_scores"] = oi.numpy(), os_.numpy()
    ii, is_ = ref.oporp_1bit_match_topk_indirect(qb, xb, 50, opos, ocnt)
    out["oporp_ind_ids"], out["oporp_ind_scores"] = ii.numpy(), is_.numpy()

    # quantizers (indexing/quantize.py)
    xq = gi.quantize_inputs()
    codes, scales = quantize_int8(xq)
    out["q8_codes"], out["q8_scales"] = codes.numpy(), scales.numpy()
    xs = gi.simhash_inputs()
    bits, r = quantize_simhash_1bit(xs, 256, seed=0)
    out["simhash_bits"], out["simhash_R"] = bits.numpy(), r.numpy()

    # SWAR popcount (functional.py:158-170)
    pc_in = torch.tensor([0, 1, 2, 3, -1, 0x5555555555555555, -(2**63)], dtype=torch.int64)
    out["popcount_in"], out["popcount_out"] = pc_in.numpy(), popcount_int64(pc_in).numpy()

    np.savez_compressed(HERE / "golden.npz", **out)
    print("wrote", HERE / "golden.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
