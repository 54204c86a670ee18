"""Builds ``oracle/_c/liboracle.so`` from ``oracle/c/*.c`` with gcc (test
infrastructure; run by ``__graft_entry__.build()`` and on first use)."""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_c" / "liboracle.so"


def build() -> Path:
    OUT.parent.mkdir(exist_ok=True)
    srcs = sorted(str(p) for p in (HERE / "c").glob("*.c"))
    stale = not OUT.exists() or any(Path(s).stat().st_mtime > OUT.stat().st_mtime for s in srcs)
    if stale:
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-shared", "-fPIC", "-o", str(OUT), *srcs, "-lm"],
                       check=True)
    return OUT


if __name__ == "__main__":
    print(build())
