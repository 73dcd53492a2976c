"""Host-side behaviour of the drop-in runtime (no GPU needed)."""
from __future__ import annotations

import pytest
import torch

from guass_b200 import cuda_field
from guass_b200.cuda_field import contracts


def test_public_names_match_reference_package():
    for name in ("gaussian_field_train", "gaussian_field_reference", "gaussian_field_forward_reference",
                 "load_extension", "STAGE0_THRESHOLDS", "TENSOR_CONTRACT", "SAVED_TENSOR_SPEC",
                 "NON_DIFFERENTIABLE_ARGS", "CUDA_FIELD_EXTENSION_NAME", "build_instructions"):
        assert hasattr(cuda_field, name), name
    assert contracts.STAGE0_THRESHOLDS.default_sigma_multiplier == 3.0


def test_extension_has_reference_methods():
    ext = cuda_field.load_extension()
    for m in ("gaussian_field_forward", "gaussian_field_backward", "gaussian_field_backward_reference"):
        assert callable(getattr(ext, m))


def _cpu_inputs(k=4):
    return (torch.linspace(-1, 1, 8), torch.linspace(-1, 1, 9), torch.zeros(k, 2), torch.zeros(k, 3),
            torch.zeros(k, 1))


def test_forward_rejects_cpu_tensors_like_torch_check():
    ext = cuda_field.load_extension()
    with pytest.raises(RuntimeError, match="row_coords must be a CUDA tensor"):
        ext.gaussian_field_forward(*_cpu_inputs(), 32, 32, 3.0, False, 80.0)


def test_backward_rejects_cpu_tensors_like_torch_check():
    ext = cuda_field.load_extension()
    row, col, mu, chol, amp = _cpu_inputs()
    with pytest.raises(RuntimeError, match="grad_delta must be a CUDA tensor"):
        ext.gaussian_field_backward(torch.zeros(72), row, col, mu, chol, amp, torch.zeros(2, dtype=torch.int64),
                                    torch.zeros(0, dtype=torch.int64), 32, 32, 3.0, False, 80.0)


def test_reference_only_guard():
    row, col, mu, chol, amp = _cpu_inputs()
    mu.requires_grad_(True)
    with pytest.raises(RuntimeError, match="validation-only"):
        cuda_field.gaussian_field_reference(row_coords=row, col_coords=col, mu=mu, chol_raw=chol, amp=amp,
                                            tile_out=32, tile_in=32, sigma_multiplier=3.0)
