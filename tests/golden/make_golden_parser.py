"""Regenerates ``tests/golden/golden_parser.npz``: SilverTorch's expression parser
``st.parse_expression_query_batch`` (silvertorch/ops/csrc/expression_query_parser.cpp:395-430,
plan encoding bloom_index_util.cpp:27-127), run by the REFERENCE's own CPU build:

    python oracle/build_ref.py <reference checkout>
    python tests/golden/make_golden_parser.py

Each case is a batch of expressions with a ``bloom_hash_k`` and ``max_sub_queries``: the
parser's ``max_stack_size``, its data bytes and its eight offsets a plan. The batches cover
every token form of the grammar (keywords and symbols, negative values, weights, nesting, the
empty match-all expression) and AND / OR chains around the ``max_sub_queries`` batching.

``ERRORS`` lists inputs the parser's checks reject (``TORCH_CHECK`` in the tokenizer and the
plan builder, expression_query_parser.cpp:94, 151, 187-193, 286-292, 318-358, and ``std::stoll``
out of range). They are not run here: this CPU build of the reference ends the process with a
segmentation fault whenever one of its checks throws, so the rejections are pinned by reading
those checks.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

BASE = [
    "42:100",
    "42:100:0.5",
    "1:100 AND 2:200",
    "1:100 & 2:200",
    "1:100 OR 2:200",
    "1:100 | 2:200",
    "NOT 3:300",
    "!3:300",
    "(1:100 AND 2:200) OR NOT 3:300",
    "(1:100 & 2:200) | !(3:300 & 4:400:0.8)",
    "1:10 OR 2:20 AND NOT 3:30",
    "1:10 OR (2:20 AND (NOT 3:30))",
    "",
    "-5:-7",
    "7:-1:3",
    "  12:34   AND\t56:78 ",
    "!!1:2",
    "NOT NOT NOT 1:2",
    "((((1:1))))",
    "(1:1 OR 2:2) AND (3:3 OR 4:4) AND NOT (5:5 OR 6:6 OR 7:7)",
    "0:0",
    "9223372036854775807:-9223372036854775808",
]


def chain(op: str, n: int, base: int = 0) -> str:
    return f" {op} ".join(f"{base + i}:{i * 3}" for i in range(n))


CHAINS = [chain(op, n) for op in ("AND", "OR") for n in range(2, 12)]
MIXED = [
    f"({chain('AND', 6)}) OR ({chain('AND', 4, 50)}) OR NOT ({chain('OR', 7, 90)})",
    " | ".join(f"({chain('&', 3, 10 * i)})" for i in range(8)),
]

CASES = [
    (BASE, 7, 5),
    (BASE, 1, 5),
    (BASE, 3, 2),
    (CHAINS + MIXED, 7, 5),
    (CHAINS + MIXED, 7, 1),
    (CHAINS + MIXED, 2, 2),
    (CHAINS + MIXED, 7, 3),
    (CHAINS + MIXED, 7, 0),
    (CHAINS + MIXED, 5, -1),
    (CHAINS, 7, 100),
]

ERRORS = [
    "1:2 AND",
    "1:2 3:4",
    "(1:2",
    "1:2)",
    "1",
    "1:",
    ":2",
    "1.5:2",
    "1:2.5",
    "1:2:x",
    "1:2 XOR 3:4",
    "and 1:2",
    "1:2 @ 3:4",
    "NOT",
    "()",
    "1:2:",
    "- 1:2",
    "1:2.3.4",
    "   ",
    "9223372036854775808:1",
]


def main() -> None:
    torch.ops.load_library(str(HERE.parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"))
    st = torch.ops.st
    out = {}
    meta = []
    for ci, (exprs, hash_k, max_sub) in enumerate(CASES):
        ks = torch.ones(len(exprs), dtype=torch.int64)
        stack, (data, offsets) = st.parse_expression_query_batch(exprs, ks, hash_k, True, max_sub)
        stack_only, (d0, o0) = st.parse_expression_query_batch(exprs, ks, hash_k, False, max_sub)
        assert stack_only == stack and d0.numel() == 0 and o0.numel() == 0
        out[f"c{ci}_data"] = data.numpy().view(np.int8)
        out[f"c{ci}_offsets"] = offsets.numpy()
        out[f"c{ci}_stack"] = np.int64(stack)
        meta.append({"expressions": exprs, "hash_k": hash_k, "max_sub_queries": max_sub})
    out["meta"] = np.array(json.dumps({"cases": meta, "rejected": ERRORS}))
    np.savez_compressed(HERE / "golden_parser.npz", **out)
    print("wrote", HERE / "golden_parser.npz", len(CASES), "cases")


if __name__ == "__main__":
    main()
