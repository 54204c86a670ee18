"""Builds ``libretrieve_b200.so`` in-tree with nvcc for sm_100a.

``python -m retrieve_b200.build`` (or ``build()``) compiles every ``csrc/*.cu``
(nvcc) and ``csrc/*.cpp`` (host code, the C++ compiler) into one shared library
next to this file. The library exports only the
``extern "C"`` entry points declared in ``include/retrieve_b200.h``; it links
the CUDA runtime statically so that the only runtime dependency is the driver.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libretrieve_b200.so"
BUILD_DIR = ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-DRB_BUILD",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-DRB_BUILD"]


def cxx_path() -> str:
    for cand in (os.environ.get("CXX"), shutil.which("g++"), shutil.which("c++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no C++ compiler found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), ROOT / "include" / "retrieve_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles every stale translation unit (in parallel) and links the library."""
    from concurrent.futures import ThreadPoolExecutor

    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    objs, cmds = [], []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if not _stale(obj, src) and not ptxas_verbose:
            continue
        if src.suffix == ".cpp":
            cmd = [cxx_path(), *CXX_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
        else:
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
    workers = max(1, min(len(cmds), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        for done in pool.map(lambda c: subprocess.run(c, check=True), cmds):
            pass
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv)
