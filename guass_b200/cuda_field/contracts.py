"""Tensor and tolerance contracts of the cuda_field boundary.

Same names and values as gaussian_peft/cuda_field/contracts.py:9-66, so code
that imports them from the reference package finds them here too.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True, slots=True)
class CudaFieldStage0Thresholds:
    default_sigma_multiplier: float = 3.0
    default_forward_mean_abs_error_max: float = 3e-3
    default_forward_max_abs_error_max: float = 2e-2
    default_backward_mean_abs_error_max: float = 2e-3
    default_backward_max_abs_error_max: float = 2e-2
    partial_grad_bytes_limit: int = 256 * 1024 * 1024
    occupancy_imbalance_ratio: float = 4.0
    occupancy_max_count_floor: int = 64
    tile_work_p95_over_p50_limit: float = 3.0


@dataclass(frozen=True, slots=True)
class CudaFieldTensorContract:
    row_coords: str = "shape=[out_features], dtype=float32, device=cuda, contiguous"
    col_coords: str = "shape=[in_features], dtype=float32, device=cuda, contiguous"
    mu: str = "shape=[K, 2], dtype=float32, device=cuda, contiguous"
    chol_raw: str = "shape=[K, 3], dtype=float32, device=cuda, contiguous"
    amp: str = "shape=[K, 1], dtype=float32, device=cuda, contiguous"
    tile_ptr: str = "shape=[num_tiles + 1], dtype=int32 or int64, device=cuda, contiguous"
    gaussian_ids_sorted: str = "shape=[num_pairs], dtype=int32 or int64, device=cuda, contiguous"
    delta: str = "shape=[out_features * in_features], dtype=float32, device=cuda, contiguous"


@dataclass(frozen=True, slots=True)
class CudaFieldSavedTensorSpec:
    mu: str = "mu"
    chol_raw: str = "chol_raw"
    amp: str = "amp"
    row_coords: str = "row_coords"
    col_coords: str = "col_coords"
    tile_ptr: str = "tile_ptr"
    gaussian_ids_sorted: str = "gaussian_ids_sorted"


@dataclass(frozen=True, slots=True)
class CudaFieldNonDifferentiableArgs:
    tile_out: str = "tile_out"
    tile_in: str = "tile_in"
    sigma_multiplier: str = "sigma_multiplier"
    normalize: str = "normalize"
    clamp_quad: str = "clamp_quad"


STAGE0_THRESHOLDS = CudaFieldStage0Thresholds()
TENSOR_CONTRACT = CudaFieldTensorContract()
SAVED_TENSOR_SPEC = CudaFieldSavedTensorSpec()
NON_DIFFERENTIABLE_ARGS = CudaFieldNonDifferentiableArgs()
