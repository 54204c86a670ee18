"""Builds the REFERENCE's own SilverTorch CPU ops (Meta's code as adapted in
rmnigm/retrieve) into ``oracle/_ref/`` — test infrastructure, used only to make
golden fixtures in the build container:

    python oracle/build_ref.py <reference checkout>
    python oracle/build_ref.py <reference checkout> --cuda

With ``--cuda`` the reference's CUDA kernels (its ``*_cuda.cu`` files; CUB from the CUDA
toolkit) are compiled for sm_100a beside the CPU ones into
``oracle/_ref/silvertorch_ref_cuda/silvertorch_ref_cuda.so``: the reference's own GPU
``st::search``, which ``bench.py --impl reference --workload ivf`` times on the same box as
this library's (in a process of its own: both libraries define the ``st`` schemas).

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


CUDA_SOURCES = [
    "bloom_index_search_cuda.cu",
    "bloom_indexer_cuda.cu",
    "expression_query_parser_cuda.cu",
    "faster_repeat_interleave.cu",
    "fork_search_cuda.cu",
    "fresh_index_post_processing_cuda.cu",
    "fused_kmean_ann_cuda.cu",
    "is_topk_cuda.cu",
]
CUDA_LIB = OUT / "silvertorch_ref_cuda" / "silvertorch_ref_cuda.so"


def build_cuda(reference: str | Path):
    import os

    from torch.utils import cpp_extension

    csrc = Path(reference) / "silvertorch" / "silvertorch" / "ops" / "csrc"
    out = CUDA_LIB.parent
    out.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    return cpp_extension.load(
        name="silvertorch_ref_cuda",
        sources=[str(csrc / s) for s in SOURCES + CUDA_SOURCES],
        extra_include_paths=[str(csrc)],
        extra_cflags=["-O2"],
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a", "--expt-relaxed-constexpr"],
        build_directory=str(out),
        is_python_module=False,
        verbose=False,
    )


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
    if len(sys.argv) not in (2, 3) or (len(sys.argv) == 3 and sys.argv[2] != "--cuda"):
        raise SystemExit("usage: python oracle/build_ref.py <reference checkout> [--cuda]")
    if len(sys.argv) == 3:
        build_cuda(sys.argv[1])
        print("built", CUDA_LIB)
    else:
        build(sys.argv[1])
        print("built into", OUT)
