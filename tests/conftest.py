"""Shared pytest setup.

Markers: ``gpu`` tests need a CUDA device (a B200) and call the product path
through libgfield's C ABI; everything else runs on the CPU.  The in-tree
library and the C oracle are (re)built here if their sources are newer.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; runs the CUDA product path")
    from guass_b200 import _build
    import oracle

    _build.build()
    oracle.build()


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
