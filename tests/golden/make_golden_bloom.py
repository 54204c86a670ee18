"""Regenerates ``tests/golden/golden_bloom.npz`` with the REFERENCE's own
SilverTorch CPU ops (built from the read-only checkout by
``oracle/build_ref.py`` into ``oracle/_ref/``):

    python oracle/build_ref.py <reference checkout>
    python tests/golden/make_golden_bloom.py

A one-bundle, 64-bit-per-doc index (``bloom_index_build`` with b_multiplier so
that max_terms * k * b_multiplier = 64) over config-3 style attributes, and
``bloom_index_search_batch`` masks for expressions of the reference's query DSL
(silvertorch/silvertorch/ops/csrc/EXPRESSION_SYNTAX.md). They pin the oracle's
hash, bit positions, item-word layout and predicate evaluation.
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
    lib = HERE.parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"
    torch.ops.load_library(str(lib))
    st = torch.ops.st
    n = 1500
    attrs = gi.zipf_attrs(n, seed=21)  # [N, 8]
    c = attrs.shape[1]
    feature_ids = torch.arange(c, dtype=torch.int32)
    offsets = torch.arange(n * c + 1, dtype=torch.int64)
    values = attrs.reshape(-1).contiguous()
    k = 3
    b_mult = 64.0 / (c * k) + 1e-6
    bloom_index, bundle_offsets = st.bloom_index_build(feature_ids, offsets, values, b_mult, k, False)
    assert bundle_offsets.tolist() == [0, 64], bundle_offsets
    ks = torch.ones(len(gi.BLOOM_EXPRESSIONS), dtype=torch.int64)
    _, (data, poffs) = st.parse_expression_query_batch(list(gi.BLOOM_EXPRESSIONS), ks, 7, True, 5)
    masks = st.bloom_index_search_batch(bloom_index, bundle_offsets, data, poffs, k, 7, True)
    np.savez_compressed(
        HERE / "golden_bloom.npz",
        attrs=attrs.numpy(),
        bloom_index=bloom_index.numpy(),
        masks=np.packbits(masks[:, :n].numpy().astype(bool), axis=1),
        n=np.array(n),
    )
    print("wrote", HERE / "golden_bloom.npz", tuple(bloom_index.shape), tuple(masks.shape))


if __name__ == "__main__":
    main()
