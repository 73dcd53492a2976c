"""Host side of the densify-statistics tracker (guass_b200.stats)."""
from __future__ import annotations

import inspect
import sys

import pytest
import torch

from guass_b200.stats import BatchedStatsTracker


def test_cuda_only_no_cpu_path():
    with pytest.raises(RuntimeError, match="needs a CUDA device"):
        BatchedStatsTracker().register_layer("a", 8, "cpu")
    with pytest.raises(ValueError, match="float32"):
        BatchedStatsTracker().register_layer("a", 8, "cuda", dtype=torch.float64)


def test_interface_matches_reference_tracker():
    from conftest import REFERENCE_ROOT as ref_root
    if ref_root not in sys.path:
        sys.path.append(ref_root)
    stats = pytest.importorskip("gaussian_peft.controllers.stats")
    ref = stats.GaussianStatsTracker
    for name, fn in inspect.getmembers(ref, inspect.isfunction):
        if name.startswith("_"):
            continue
        ours = getattr(BatchedStatsTracker, name, None)
        assert ours is not None, name
        assert list(inspect.signature(ours).parameters) == list(inspect.signature(fn).parameters), name
