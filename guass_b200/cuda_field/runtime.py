"""Autograd runtime with the reference runtime's public functions.

Same entry points, argument order and return protocol as
gaussian_peft/cuda_field/runtime.py:11-345, on top of this package's
extension object.  The forward saves the reference's seven tensors
(row_coords, col_coords, mu, chol_raw, amp, tile_ptr, gaussian_ids_sorted;
runtime.py:148-156) and the backward returns gradients for mu, chol_raw and amp
only (runtime.py:192-203).
"""
from __future__ import annotations

import torch
from torch import Tensor

from guass_b200.cuda_field import loader as _loader


def load_extension(*, verbose: bool = False):
    """Module-level indirection so tests and integrations can substitute it."""
    return _loader.load_extension(verbose=verbose)


class _FieldFunctionBase(torch.autograd.Function):
    _backward_method = "gaussian_field_backward"

    @staticmethod
    def forward(ctx, row_coords: Tensor, col_coords: Tensor, mu: Tensor, chol_raw: Tensor, amp: Tensor,
                tile_out: int, tile_in: int, sigma_multiplier: float, normalize: bool,
                clamp_quad: float | None) -> Tensor:
        ext = load_extension(verbose=False)
        delta, tile_ptr, gaussian_ids_sorted = ext.gaussian_field_forward(
            row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in, sigma_multiplier, normalize, clamp_quad)
        ctx.save_for_backward(row_coords, col_coords, mu, chol_raw, amp, tile_ptr, gaussian_ids_sorted)
        ctx.field_args = (tile_out, tile_in, sigma_multiplier, normalize, clamp_quad)
        return delta

    @classmethod
    def _backward(cls, ctx, grad_delta: Tensor):
        ext = load_extension(verbose=False)
        saved = ctx.saved_tensors
        grads = getattr(ext, cls._backward_method)(grad_delta.contiguous(), *saved, *ctx.field_args)
        d_mu, d_chol_raw, d_amp = grads
        return None, None, d_mu, d_chol_raw, d_amp, None, None, None, None, None


class GaussianFieldCudaTrainFunction(_FieldFunctionBase):
    """The training path (runtime.py:107-203): explicit CUDA backward.

    With this package's extension the binning stays in the library's
    shared-id form (``train_forward`` / ``train_backward``): the same kernels
    and results, but the pair count travels to the host asynchronously, so a
    model's layers render without a synchronisation each.  The saved state is
    then the reference's seven tensors with the device pair count appended
    (and its host copy on the context).  Any other extension object (e.g. the reference's
    own) is driven through the reference protocol."""

    @staticmethod
    def forward(ctx, row_coords: Tensor, col_coords: Tensor, mu: Tensor, chol_raw: Tensor, amp: Tensor,
                tile_out: int, tile_in: int, sigma_multiplier: float, normalize: bool,
                clamp_quad: float | None) -> Tensor:
        ext = load_extension(verbose=False)
        ctx.field_args = (tile_out, tile_in, sigma_multiplier, normalize, clamp_quad)
        ctx.shared_ids = hasattr(ext, "train_forward")
        if not ctx.shared_ids:
            delta, tile_ptr, ids = ext.gaussian_field_forward(row_coords, col_coords, mu, chol_raw, amp, tile_out,
                                                              tile_in, sigma_multiplier, normalize, clamp_quad)
            ctx.save_for_backward(row_coords, col_coords, mu, chol_raw, amp, tile_ptr, ids)
            return delta
        delta, tile_ptr, ids, pair_base, ctx.probe = ext.train_forward(row_coords, col_coords, mu, chol_raw, amp,
                                                                       tile_out, tile_in, sigma_multiplier, normalize,
                                                                       clamp_quad)
        ctx.save_for_backward(row_coords, col_coords, mu, chol_raw, amp, tile_ptr, ids, pair_base)
        return delta

    @staticmethod
    def backward(ctx, grad_delta: Tensor):
        if not ctx.shared_ids:
            return GaussianFieldCudaTrainFunction._backward(ctx, grad_delta)
        ext = load_extension(verbose=False)
        d_mu, d_chol_raw, d_amp = ext.train_backward(grad_delta.contiguous(), *ctx.saved_tensors, *ctx.field_args,
                                                     probe=ctx.probe)
        return None, None, d_mu, d_chol_raw, d_amp, None, None, None, None, None


class GaussianFieldCudaReferenceFunction(_FieldFunctionBase):
    """Validation path (runtime.py:11-104); calls the extension's
    ``gaussian_field_backward_reference``."""

    _backward_method = "gaussian_field_backward_reference"

    @staticmethod
    def backward(ctx, grad_delta: Tensor):
        return GaussianFieldCudaReferenceFunction._backward(ctx, grad_delta)


def gaussian_field_forward_reference(*, row_coords: Tensor, col_coords: Tensor, mu: Tensor, chol_raw: Tensor,
                                     amp: Tensor, tile_out: int, tile_in: int, sigma_multiplier: float,
                                     normalize: bool = False, clamp_quad: float | None = 80.0,
                                     verbose_build: bool = False) -> tuple[Tensor, Tensor, Tensor]:
    ext = load_extension(verbose=verbose_build)
    return tuple(ext.gaussian_field_forward(row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in,
                                            sigma_multiplier, normalize, clamp_quad))


def gaussian_field_reference(*, row_coords: Tensor, col_coords: Tensor, mu: Tensor, chol_raw: Tensor, amp: Tensor,
                             tile_out: int, tile_in: int, sigma_multiplier: float, normalize: bool = False,
                             clamp_quad: float | None = 80.0, allow_reference_backward: bool = False) -> Tensor:
    # runtime.py:250-258
    if not allow_reference_backward and (mu.requires_grad or chol_raw.requires_grad or amp.requires_grad):
        raise RuntimeError(
            "gaussian_field_reference is validation-only. Set allow_reference_backward=True only for explicit "
            "gradient alignment checks; do not use this path as a training backend.")
    return GaussianFieldCudaReferenceFunction.apply(row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in,
                                                    sigma_multiplier, normalize, clamp_quad)


def gaussian_field_train(*, row_coords: Tensor, col_coords: Tensor, mu: Tensor, chol_raw: Tensor, amp: Tensor,
                         tile_out: int, tile_in: int, sigma_multiplier: float, normalize: bool = False,
                         clamp_quad: float | None = 80.0) -> Tensor:
    return GaussianFieldCudaTrainFunction.apply(row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in,
                                                sigma_multiplier, normalize, clamp_quad)


def gaussian_field_cuda_field_stage2_validation(*, row_coords: Tensor, col_coords: Tensor, mu: Tensor,
                                                chol_raw: Tensor, amp: Tensor, tile_out: int, tile_in: int,
                                                sigma_multiplier: float, normalize: bool = False,
                                                clamp_quad: float | None = 80.0, verbose_build: bool = False):
    """Forward plus binning metadata (runtime.py:300-345)."""
    delta, tile_ptr, ids = gaussian_field_forward_reference(
        row_coords=row_coords, col_coords=col_coords, mu=mu, chol_raw=chol_raw, amp=amp, tile_out=tile_out,
        tile_in=tile_in, sigma_multiplier=sigma_multiplier, normalize=normalize, clamp_quad=clamp_quad,
        verbose_build=verbose_build)
    metadata = {
        "execution_mode": "cuda_field_stage2_validation",
        "tile_ptr": tile_ptr,
        "gaussian_ids": ids,
        "gaussian_ids_sorted": ids,
        "per_tile_counts": tile_ptr[1:] - tile_ptr[:-1],
        "tiles_touched": torch.full((mu.size(0),), -1, device=mu.device, dtype=torch.int64),
        "num_tile_rows": float((row_coords.numel() + tile_out - 1) // tile_out),
        "num_tile_cols": float((col_coords.numel() + tile_in - 1) // tile_in),
        "accumulate_backend": "cuda_field_stage2_validation",
    }
    return delta, metadata
