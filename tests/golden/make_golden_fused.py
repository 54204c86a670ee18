"""Regenerates ``tests/golden/golden_fused.npz``: the REFERENCE's CPU scorer
``st.fused_kmean_ann`` (silvertorch/ops/csrc/fused_kmean_ann.cpp:86-228) with its two
options the adapter's official path leaves unset, ``per_embedding_scale`` (a per-doc fp16
divisor) and ``filtering_bit_index`` (query row -> mask row), and on float embeddings:

    python oracle/build_ref.py <reference checkout>
    python tests/golden/make_golden_fused.py

Codes are small (|dot| <= 1024), where the CPU scorer's ``Half(float(dot) / scale)`` and the CUDA
scorer's ``Half(float(Half(dot)) / float(scale))`` (index_mm_helpers.cuh:49-56, the dot first
rounded to fp16) agree: the fp16 rounding of an integer below 2048 is exact. The CPU scorer reads
the mask low bit first, the CUDA scorer high bit first (bloom_index_util.cuh:137-147): the fixture
stores the boolean mask, the CPU run gets it packed low bit first.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def pack_low_first(mask: torch.Tensor) -> torch.Tensor:
    r, n = mask.shape
    w = (n + 63) // 64
    padded = torch.zeros(r, w * 64, dtype=torch.bool)
    padded[:, :n] = mask
    bits = padded.view(r, w, 64).to(torch.int64)
    return (bits << torch.arange(64, dtype=torch.int64)).sum(-1)  # wraps into int64 like the C++ words


def main() -> None:
    torch.ops.load_library(str(HERE.parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"))
    st = torch.ops.st
    g = torch.Generator().manual_seed(23)
    n_lists, d, b, p = 24, 64, 12, 4
    sizes = torch.randint(0, 120, (n_lists,), generator=g)
    offsets = torch.cat([torch.zeros(1, dtype=torch.int64), sizes.cumsum(0)])
    n = int(offsets[-1])
    codes = torch.randint(-4, 5, (n, d), generator=g).to(torch.int8)
    q = torch.randint(-4, 5, (b, d), generator=g).to(torch.int8)
    probe = torch.stack([torch.randperm(n_lists, generator=g)[:p] for _ in range(b)])
    lengths = sizes[probe]
    width = int(lengths.sum(1).max())
    scale = (torch.rand(n, generator=g) * 4 + 0.05).to(torch.float16)
    scale[:8] = torch.tensor([1, 2, 0.5, 4, 0.25, 3, 0.1, 7], dtype=torch.float16)
    rows = 5
    mask = torch.rand(rows, n, generator=g) < 0.6
    mask_index = torch.randint(0, rows, (b,), generator=g)
    args = (offsets, probe, lengths, codes, q, width)
    out = {"offsets": offsets.numpy(), "probe": probe.numpy(), "lengths": lengths.numpy(), "codes": codes.numpy(),
           "q": q.numpy(), "width": np.int64(width), "scale": scale.numpy(), "mask": mask.numpy(),
           "mask_index": mask_index.numpy()}
    cases = {
        "scaled": dict(per_embedding_scale=scale),
        "scaled_div": dict(per_embedding_scale=scale, divisor_for_int8=16),
        "index_i32": dict(filtering_bit_mask=pack_low_first(mask), filtering_bit_index=mask_index),
        "index_scaled": dict(filtering_bit_mask=pack_low_first(mask), filtering_bit_index=mask_index,
                             per_embedding_scale=scale, invalid_index_value=-5),
    }
    for name, kw in cases.items():
        raw, idx = st.fused_kmean_ann(*args, **kw)
        out[f"{name}_raw"] = raw.numpy()
        out[f"{name}_idx"] = idx.numpy()
    # float embeddings with entries in {-1, 0, 1}: every partial dot is a small integer, exact in
    # fp32 and fp16, so the CPU scorer's fp64 dot and the CUDA scorer's rounded chains agree. (bf16:
    # the CPU scorer fails to fill its output with -FLT_MAX, which bf16 cannot hold —
    # fused_kmean_ann.cpp:151-156, "value cannot be converted to type c10::BFloat16 without
    # overflow"; the CUDA scorer fills with the lowest finite bf16, 0xff7f.)
    tern_x = torch.randint(-1, 2, (n, d), generator=g)
    tern_q = torch.randint(-1, 2, (b, d), generator=g)
    out["tern_x"], out["tern_q"] = tern_x.to(torch.int8).numpy(), tern_q.to(torch.int8).numpy()
    for name, dt in (("f32", torch.float32), ("f16", torch.float16)):
        raw, idx = st.fused_kmean_ann(offsets, probe, lengths, tern_x.to(dt), tern_q.to(dt), width,
                                      filtering_bit_mask=pack_low_first(mask), filtering_bit_index=mask_index,
                                      invalid_index_value=-2)
        assert raw.dtype == dt
        out[f"{name}_raw"] = raw.float().numpy()
        out[f"{name}_idx"] = idx.numpy()
    np.savez_compressed(HERE / "golden_fused.npz", **out)
    print("wrote", HERE / "golden_fused.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
