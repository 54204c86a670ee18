"""Regenerates ``tests/golden/golden_ivf.npz``: SilverTorch's IVF probe + int8
search (``st::search`` semantics) computed by the REFERENCE's own code, on CPU:

    python oracle/build_ref.py <reference checkout>      # builds oracle/_ref/
    PYTHONPATH=<reference>/retrieve/src python tests/golden/make_golden_ivf.py

Per case, the reference's adapter epilogue ``official_probe_score``
(retrieve/src/retrieve/ops/official/adapter.py:433-478: ``quantize_int8`` of the
query, the raw scorer, ``torch.topk`` on the raw scores, ``sort_perm`` and the
two-multiply dequantization of the winners) runs over the reference's CPU
scorer ``st.fused_kmean_ann`` (silvertorch/ops/csrc/fused_kmean_ann.cpp:86-214,
compiled from the checkout into ``oracle/_ref/``), on the int32 path, on the
fp16 path (``default_divisor(D)``) and with a full-``N`` filter mask. The
scorer's raw ``(scores, indices)`` rows are stored too.

Two CPU-versus-CUDA differences are handled here so that the fixture holds
what the CUDA op returns:

* ``quantize_int8`` on a CPU tensor divides ``abs_max`` by 127; on a CUDA tensor
  (and in the op's query prep) it multiplies by fp32(1/127). Only query rows
  whose two scales agree are kept, so the CPU run gives the device scores.
* The CPU scorer reads the filter mask low bit first, the CUDA scorer high bit
  first. The fixture stores the boolean mask; the CPU run gets it packed low bit
  first, the oracle (like the CUDA op) packs it high bit first.

The CPU scorer writes a row's positions in probe order, the CUDA scorer in its
warp-prefix-then-remainder order, so tied raw scores may keep different ids:
the fixture is compared with scores exact and ids up to ties, as the
reference's own parity test does (retrieve/tests/parity/test_official.py:211-217).
Case shapes follow that test's grid (test_official.py:248-262), plus a
tie-heavy table (four distinct code rows).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

# (n_lists, max_size, n_probe, d, k, b, ties)
CASES = [
    (16, 64, 4, 64, 8, 16, False),
    (32, 96, 8, 128, 32, 16, False),
    (32, 64, 8, 96, 16, 1, False),
    (32, 90, 8, 128, 32, 16, False),
    (32, 90, 8, 192, 32, 16, False),
    (16, 90, 8, 768, 32, 4, False),
    (64, 200, 16, 128, 100, 8, True),
]


def layout(g: torch.Generator, b: int, n_lists: int, max_size: int, n_probe: int):
    """A cluster-sorted table: sizes in [0, max_size] (multiples of 32 and not), CSR offsets,
    a random sorted-position -> item-id permutation, and ``n_probe`` distinct clusters per row."""
    sizes = torch.randint(0, max_size + 1, (n_lists,), generator=g, dtype=torch.int64)
    sizes[0] = max_size // 32 * 32  # one cluster of whole warps
    sizes[1] = 0  # one empty cluster
    offsets = torch.cat([sizes.new_zeros(1), sizes.cumsum(0)])
    n = int(offsets[-1])
    sort_perm = torch.randperm(n, generator=g, dtype=torch.int64)
    probe = torch.rand(b, n_lists, generator=g).argsort(1)[:, :n_probe].contiguous()
    width = int(sizes[probe].sum(1).max())
    return sizes, offsets, sort_perm, probe, width


def device_scale_rows(q: torch.Tensor) -> torch.Tensor:
    """Rows whose CPU scale (``abs_max / 127``) equals the CUDA one (``abs_max * fp32(1/127)``)."""
    am = q.abs().amax(1).clamp(min=1e-8)
    return (am / 127.0) == (am * torch.tensor(1.0 / 127.0, dtype=torch.float32))


def main() -> None:
    torch.ops.load_library(str(HERE.parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"))
    import retrieve.ops.official as of
    from retrieve.indexing.quantize import quantize_int8, quantize_int8_global
    from retrieve.ops.official import adapter

    of._LOAD_MEMO[:] = [torch.ops.st]  # the checkout's CPU scorer, registered above
    out: dict[str, np.ndarray] = {}
    for ci, (n_lists, max_size, n_probe, d, k, b, ties) in enumerate(CASES):
        g = torch.Generator().manual_seed(100 + ci)
        sizes, offsets, sort_perm, probe, width = layout(g, b, n_lists, max_size, n_probe)
        n = int(offsets[-1])
        if ties:
            base = torch.randn(4, d, generator=g)
            embs = base[torch.randint(0, 4, (n,), generator=g)]
        else:
            embs = torch.randn(n, d, generator=g)
        codes, gs = quantize_int8_global(embs)
        gst = torch.tensor(gs, dtype=torch.float32)
        q = torch.randn(4 * b, d, generator=g)
        q = q[device_scale_rows(q)][:b].contiguous()
        assert q.shape[0] == b
        args = (q, probe, offsets, sizes, codes, sort_perm, gst, k, width)
        ids32, sc32 = adapter.official_probe_score(*args, score_path="int32")
        div = adapter.default_divisor(d)
        ids16, sc16 = adapter.official_probe_score(*args, score_path="fp16", divisor=div)
        mask = torch.rand(b, n, generator=g) < 0.5
        low_first = adapter.pack_mask(mask, "low_first")
        idsm, scm = adapter.official_probe_score(*args, score_path="int32", filtering_bit_mask=low_first)
        q_codes, _ = quantize_int8(q)
        raw, idx = adapter.fused_scores(q_codes, probe, offsets, sizes, codes, width)
        p = f"c{ci}_"
        out.update({
            p + "shape": np.array([n_lists, max_size, n_probe, d, k, b, width, div, int(ties)], dtype=np.int64),
            p + "query": q.numpy(), p + "probe": probe.numpy(), p + "offsets": offsets.numpy(),
            p + "sizes": sizes.numpy(), p + "codes": codes.numpy(), p + "sort_perm": sort_perm.numpy(),
            p + "gs": gst.numpy(), p + "mask": mask.numpy(),
            p + "ids32": ids32.numpy(), p + "sc32": sc32.numpy(),
            p + "ids16": ids16.numpy(), p + "sc16": sc16.numpy(),
            p + "idsm": idsm.numpy(), p + "scm": scm.numpy(),
            p + "raw": raw.numpy(), p + "idx": idx.numpy(),
        })  # fmt: skip
    np.savez_compressed(HERE / "golden_ivf.npz", **out)
    print("wrote", HERE / "golden_ivf.npz", len(CASES), "cases")


if __name__ == "__main__":
    main()
