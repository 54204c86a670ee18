"""Regenerates ``tests/golden/golden_quant.npz`` with the REFERENCE's own
quantizers and packers (retrieve/src/retrieve/indexing/quantize.py), run on CPU
tensors:

    PYTHONPATH=<reference>/retrieve/src python tests/golden/make_golden_quant.py

* ``quantize_int8_global`` (:34-52) on a table, whole and through a row
  permutation (the cluster-sorted build), and on a table holding a NaN;
* ``quantize_int8`` (:9-18) on rows holding a NaN and an infinity;
* ``_pack_signs_to_int64`` (:63-72) on values with zeros, negative zeros, NaN
  and ties at 0, and the full 1-bit builds ``quantize_simhash_1bit`` (:148-164)
  and ``quantize_oporp_1bit`` (:108-124, k_bits = D) with their query-side
  projections.

On CPU tensors the scales are a division by 127; the CUDA form multiplies by
fp32(1/127) (the tests compare both). Codes and bits do not depend on it.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main() -> None:
    from retrieve.indexing import quantize as qz

    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(11)
    x = torch.randn(1000, 64, generator=g) * 3.0
    x[5, 7] = 40.0  # one element sets the global scale
    codes, scale = qz.quantize_int8_global(x)
    perm = torch.randperm(1000, generator=g)
    codes_p, scale_p = qz.quantize_int8_global(x, rows=perm)
    out.update(global_x=x.numpy(), global_codes=codes.numpy(), global_scale=np.float32(scale),
               global_perm=perm.numpy(), global_codes_perm=codes_p.numpy(), global_scale_perm=np.float32(scale_p))
    xn = x[:64].clone()
    xn[3, 2] = float("nan")
    codes_n, scale_n = qz.quantize_int8_global(xn)
    out.update(global_nan_x=xn.numpy(), global_nan_codes=codes_n.numpy(), global_nan_scale=np.float32(scale_n))

    q = torch.randn(8, 64, generator=g)
    q[1, 4] = float("nan")
    q[2, 0] = float("inf")
    qc, qs = qz.quantize_int8(q)
    out.update(q8_special_x=q.numpy(), q8_special_codes=qc.numpy(), q8_special_scales=qs.numpy())

    v = torch.randn(40, 256, generator=g)
    v[0, :64] = 0.0
    v[1, :64] = -0.0
    v[2, 10] = float("nan")
    v[3] = torch.where(v[3] > 0, 1e-45, -1e-45)  # the smallest subnormals: signs still count
    out.update(pack_values=v.numpy(), pack_words=qz._pack_signs_to_int64(v).numpy())

    embs = torch.randn(200, 128, generator=g)
    query = torch.randn(16, 128, generator=g)
    bits, r = qz.quantize_simhash_1bit(embs, 512, seed=3)
    qbits = qz.project_simhash_1bit_query(query, r)
    out.update(sim_embs=embs.numpy(), sim_query=query.numpy(), sim_r=r.numpy(), sim_bits=bits.numpy(),
               sim_qbits=qbits.numpy())
    obits, signs, operm = qz.quantize_oporp_1bit(embs, seed=5)
    oq = qz.project_oporp_1bit_query(query, signs, operm)
    out.update(oporp_bits=obits.numpy(), oporp_signs=signs.numpy(), oporp_perm=operm.numpy(), oporp_qbits=oq.numpy())
    np.savez_compressed(HERE / "golden_quant.npz", **out)
    print("wrote", HERE / "golden_quant.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
