"""Builds the REFERENCE's own SilverTorch CPU ops (Meta's code as adapted in
rmnigm/retrieve) into ``oracle/_ref/`` — test infrastructure, used only to make
golden fixtures in the build container:

    python oracle/build_ref.py <reference checkout>

The C++ sources are compiled where they lie (read-only) with torch's
``cpp_extension`` (they need the ATen headers torch ships); the library lands in
``oracle/_ref/`` (git-ignored) and registers ``torch.ops.st.*`` (CPU kernels:
bloom_index_build, bloom_index_search_batch, parse_expression_query_batch,
fused_kmean_ann, ...). Nothing in the product, the GPU tests or the bench uses it.
"""

from __future__ import annotations

import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
SOURCES = [
    "bloom_index_util.cpp",
    "bloom_indexer.cpp",
    "bloom_index_search.cpp",
    "expression_query_parser.cpp",
    "fused_kmean_ann.cpp",
    "fork_search.cpp",
    "is_topk.cpp",
    "fresh_index_post_processing.cpp",
]


def build(reference: str | Path):
    from torch.utils import cpp_extension

    csrc = Path(reference) / "silvertorch" / "silvertorch" / "ops" / "csrc"
    OUT.mkdir(exist_ok=True)
    return cpp_extension.load(
        name="silvertorch_ref_cpu",
        sources=[str(csrc / s) for s in SOURCES],
        extra_include_paths=[str(csrc)],
        extra_cflags=["-O2"],
        build_directory=str(OUT),
        is_python_module=False,
        verbose=False,
    )


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python oracle/build_ref.py <reference checkout>")
    build(sys.argv[1])
    print("built into", OUT)
