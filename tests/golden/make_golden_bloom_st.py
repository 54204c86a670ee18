"""Regenerates ``tests/golden/golden_bloom_st.npz``: SilverTorch's own bloom index,
query plans and bloom search, computed by the REFERENCE's CPU ops (built from the
read-only checkout into ``oracle/_ref/``):

    python oracle/build_ref.py <reference checkout>
    PYTHONPATH=<reference>/retrieve/src python tests/golden/make_golden_bloom_st.py

* ``st.bloom_index_build`` (silvertorch/ops/csrc/bloom_indexer.cpp:27-114) over the
  attrs in the reference's feature layout (``adapter.attrs_to_features``,
  retrieve/src/retrieve/ops/official/adapter.py:45-65), Meta's width
  (``b_multiplier`` 10, ``build_k`` 5);
* ``st.parse_expression_query_batch`` (expression_query_parser.cpp:395-430) on DSL
  expressions with AND / OR / NOT / parentheses and the empty (match-all) query, with
  7 stored hashes a term;
* ``st.bloom_index_search_batch`` (bloom_index_search.cpp:379-396) with k = 5: the
  bool mask over every doc, which ``st::search``'s bloom filter must reproduce over
  the probed docs (fork_search_cuda.cu:1301-1325: "the bloom over the probed
  clusters' columns only ... so the full path's result too"), and the packed int64
  words of the same search (``return_bool_mask=False``);
* ``st.generate_column_info_for_clusters`` (bloom_index_search.cpp:494-538) and
  ``st.bloom_index_search_batch_return_partial_response`` (:244-374) over probed
  ranges of a cluster layout of the 5000 docs: one plan a row, and 14 rows mapped
  to plans by ``query_plan_index``.

The constants are the reference's bloom gates' (retrieve/tests/parity/test_official.py:52).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
K_SEARCH, HASH_K, B_MULT = 5, 7, 10.0

EXPRESSIONS = [
    "0:3",
    "0:3 AND 1:5",
    "0:1 OR 2:7",
    "NOT 1:2",
    "(0:1 OR 0:2) AND NOT 2:3",
    "",
    "1:0 AND (2:4 OR NOT 0:9)",
    "2:11",
    "0:5 OR 1:5 OR 2:5",
    "NOT (0:0 OR 1:1)",
]


def main() -> None:
    torch.ops.load_library(str(HERE.parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"))
    from retrieve.ops.official import adapter

    st = torch.ops.st
    g = torch.Generator().manual_seed(17)
    n, c, a = 5000, 3, 2
    attrs = torch.randint(0, 12, (n, c, a), generator=g)
    attrs[torch.rand(n, c, a, generator=g) < 0.3] = -1  # ragged values, some clauses empty
    fid, foff, fval = adapter.attrs_to_features(attrs)
    index, boff = st.bloom_index_build(fid, foff, fval, B_MULT, K_SEARCH, False)
    ks = torch.ones(len(EXPRESSIONS), dtype=torch.int64)
    max_stack, (data, offsets) = st.parse_expression_query_batch(EXPRESSIONS, ks, HASH_K, True, 5)
    mask = st.bloom_index_search_batch(index, boff, data, offsets, K_SEARCH, HASH_K, True)
    assert mask.dtype == torch.bool and mask.shape[0] == len(EXPRESSIONS) and mask.shape[1] >= n
    words = st.bloom_index_search_batch(index, boff, data, offsets, K_SEARCH, HASH_K, False)
    assert words.dtype == torch.int64 and words.shape == (len(EXPRESSIONS), mask.shape[1] // 64)
    # probed ranges: a cluster layout of the n docs (sizes 0..149, cut at n), P probes a row
    ends = torch.randint(0, 150, (80,), generator=g).cumsum(0).clamp(max=n)
    coff = torch.cat([torch.zeros(1, dtype=torch.int64), ends])
    sizes = coff.diff()
    n_probe = 4
    probe = torch.randint(0, sizes.numel(), (len(EXPRESSIONS), n_probe), generator=g)
    sel_off, sel_len = coff[probe].contiguous(), sizes[probe].contiguous()
    counts, starts, first = st.generate_column_info_for_clusters(sel_off, sel_len)
    p_cumsum, p_first, p_words = st.bloom_index_search_batch_return_partial_response(
        index, boff, data, offsets, sel_off, sel_len, K_SEARCH, HASH_K)
    rows = 14
    plan_idx = torch.randint(0, len(EXPRESSIONS), (rows,), generator=g)
    probe2 = torch.randint(0, sizes.numel(), (rows, n_probe), generator=g)
    sel_off2, sel_len2 = coff[probe2].contiguous(), sizes[probe2].contiguous()
    q_cumsum, q_first, q_words = st.bloom_index_search_batch_return_partial_response(
        index, boff, data, offsets, sel_off2, sel_len2, K_SEARCH, HASH_K, plan_idx)
    out = {
        "attrs": attrs.numpy(), "bloom_index": index.numpy(), "bundle_b_offsets": boff.numpy(),
        "plan_data": data.numpy().view(np.int8), "plan_offsets": offsets.numpy(),
        "max_stack": np.int64(max_stack), "k": np.int64(K_SEARCH), "hash_k": np.int64(HASH_K),
        "mask_bits": np.packbits(mask[:, :n].numpy(), axis=1), "n": np.int64(n),
        "words": words.numpy(), "cluster_offsets": coff.numpy(), "cluster_sizes": sizes.numpy(),
        "probe": probe.numpy(), "col_counts": counts.numpy(), "col_starts": starts.numpy(),
        "col_first": first.numpy(), "p_cumsum": p_cumsum.numpy(), "p_first": p_first.numpy(),
        "p_words": p_words.numpy(), "plan_index": plan_idx.numpy(), "probe2": probe2.numpy(),
        "q_cumsum": q_cumsum.numpy(), "q_first": q_first.numpy(), "q_words": q_words.numpy(),
    }  # fmt: skip
    np.savez_compressed(HERE / "golden_bloom_st.npz", **out)
    print("wrote", HERE / "golden_bloom_st.npz", {k: np.shape(v) for k, v in out.items()})


if __name__ == "__main__":
    main()
