"""Shared pytest setup.

Markers: ``gpu`` tests need a CUDA device (a B200) and call the product path
through libgfield's C ABI; everything else runs on the CPU.  The in-tree
library and the C oracle are (re)built here if their sources are newer.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# GUASS project root with the reference sources (tests that import or build
# the reference skip when it is absent, as on the GPU box)
REFERENCE_ROOT = os.environ.get("GUASS_REFERENCE_ROOT", "/root/reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; runs the CUDA product path")
    from guass_b200 import _build
    import oracle

    _build.build_all()
    oracle.build()


# GPU modules run in this order (the others after them, test_zz_* last), so
# that under -x the core parity tests always run before the newer ones.
_GPU_ORDER = ("test_gpu_parity", "test_gpu_reference_ext", "test_gpu_properties", "test_gpu_multigpu")


def _rank(item):
    mod = item.module.__name__.rsplit(".", 1)[-1] if item.module else ""
    if mod.startswith("test_zz"):
        return len(_GPU_ORDER) + 1
    return _GPU_ORDER.index(mod) if mod in _GPU_ORDER else len(_GPU_ORDER)


def pytest_collection_modifyitems(config, items):
    import torch

    items.sort(key=_rank)  # stable: file order within a rank
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
