"""Test configuration: the ``gpu`` marker (tests that need a B200 and the built
library) and the repo root on ``sys.path`` so ``oracle`` and ``retrieve_b200``
import without installation."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libretrieve_b200.so")


# Modules run in this order after all others (a stable sort): SilverTorch's ops by how central
# they are to the search path, then the build-time tools and the end-to-end pipeline built from
# them, the reference's own modules on this library, and the no-allocation entry point's test
# last of all. Under ``-x`` a failure in one of these leaves every test before it already run.
LATE_MODULES = ("test_st_search", "test_st_bloom", "test_st_select", "test_quantizers", "test_kmeans",
                "test_ivf_pipeline", "test_dropin_reference", "test_zz_no_alloc")


def _rank(item) -> int:
    name = Path(str(item.fspath)).stem
    return LATE_MODULES.index(name) + 1 if name in LATE_MODULES else 0


def pytest_collection_modifyitems(config, items):
    import torch

    items.sort(key=_rank)
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device here")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
