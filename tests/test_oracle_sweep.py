"""Seeded sweep: the oracle against GUASS's own PyTorch path on random small
configurations (shapes, tile sizes, sigma multiplier, normalize, clamp,
scales).  Runs where the reference package is importable (the build
container); the committed golden fixtures cover the same ground elsewhere.

The torch path and the CUDA extension differ on one point: the torch path
inverts the covariance with ``torch.linalg.inv`` and no determinant floor
(gaussian_peft/kernels/covariance.py:35-38), while the CUDA extension floors
det at 1e-8 (gaussian_peft/cuda_field/csrc/forward.cu:171).  The
oracle follows the CUDA extension.  Gaussians near the floor therefore get
amplitude 0 on both sides, so that they drop out of delta and of every
gradient except their own d_amp, which is left out of the comparison; tile
binning does not depend on amp and is still compared for all of them."""
from __future__ import annotations

import math
import sys

import numpy as np
import pytest
import torch

from conftest import REFERENCE_ROOT as REF  # noqa: E402
if REF not in sys.path:
    sys.path.append(REF)
pytest.importorskip("gaussian_peft")

import oracle  # noqa: E402
from guass_b200.synthetic import make_field  # noqa: E402
from sweep_configs import draw  # noqa: E402


def _ref(f, to, ti, sigma, norm, clamp):
    from gaussian_peft.kernels.covariance import activate_cholesky
    from gaussian_peft.kernels.gaussian_field import gaussian_field

    mu = f.mu.clone().requires_grad_(True)
    chol_raw = f.chol_raw.clone().requires_grad_(True)
    amp = f.amp.clone().requires_grad_(True)
    delta, meta = gaussian_field(torch.zeros(1, 2), mu, activate_cholesky(chol_raw, eps=1e-5), amp, normalize=norm,
                                 clamp_quad=clamp, execution_mode="tiled_reference_pytorch", row_coords=f.row_coords,
                                 col_coords=f.col_coords, tile_out=to, tile_in=ti, sigma_multiplier=sigma,
                                 return_metadata=True)
    delta.backward(f.grad)
    return delta.detach().numpy(), meta["tile_ptr"].numpy(), meta["gaussian_ids"].numpy(), \
        (mu.grad.numpy(), chol_raw.grad.numpy(), amp.grad.numpy())


@pytest.mark.parametrize("seed", range(24))
def test_oracle_vs_reference_torch_random_config(seed):
    f, kw = draw(seed)
    to, ti, sigma, norm, clamp = (kw["tile_out"], kw["tile_in"], kw["sigma_multiplier"], kw["normalize"],
                                  kw["clamp_quad"])
    from gaussian_peft.kernels.covariance import activate_cholesky
    L = activate_cholesky(f.chol_raw.double(), eps=1e-5)
    det = (L[:, 0, 0] * L[:, 1, 1]).square()
    floored = (det < 4e-8).numpy()  # the 1e-8 floor with a margin for fp32 rounding of det
    if floored.any():
        f.amp = f.amp.masked_fill(torch.from_numpy(floored).view(-1, *([1] * (f.amp.dim() - 1))), 0.0)
    d, tp, ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, **kw)
    rd, rtp, rids, rg = _ref(f, to, ti, sigma, norm, clamp)
    np.testing.assert_array_equal(tp, rtp)
    for t in range(tp.size - 1):
        assert sorted(ids[tp[t]:tp[t + 1]]) == sorted(rids[tp[t]:tp[t + 1]])
    scale = max(np.abs(rd).max(), 1e-30)
    assert np.abs(d - rd).max() <= 1e-5 * scale
    g = oracle.backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tp, ids, **kw)
    keep = ~floored
    for a, b, n in zip(g, rg, ("d_mu", "d_chol_raw", "d_amp")):
        a, b = a[keep], b[keep]
        if b.size == 0:
            continue
        assert np.abs(a - b).max() <= 1e-4 * max(np.abs(b).max(), 1e-30), n


@pytest.mark.parametrize("shape", [(1, 1, 3, 32, 32), (3, 200, 4, 64, 64), (130, 1, 6, 8, 8), (5, 7, 0, 32, 32)])
def test_oracle_vs_reference_torch_degenerate_shapes(shape):
    """1x1 fields, single rows and columns, tiles larger than the field, and
    K = 0 (forward only: the reference's autograd has nothing to differentiate)."""
    out_f, in_f, k, to, ti = shape
    f = make_field(out_f, in_f, k, seed=1, log_scale_mean=math.log(0.2))
    kw = dict(tile_out=to, tile_in=ti, sigma_multiplier=3.0, normalize=False, clamp_quad=80.0)
    d, tp, ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, **kw)
    if k == 0:
        from gaussian_peft.kernels.covariance import activate_cholesky
        from gaussian_peft.kernels.gaussian_field import gaussian_field

        rd, meta = gaussian_field(torch.zeros(1, 2), f.mu, activate_cholesky(f.chol_raw, eps=1e-5), f.amp,
                                  clamp_quad=80.0, execution_mode="tiled_reference_pytorch", row_coords=f.row_coords,
                                  col_coords=f.col_coords, tile_out=to, tile_in=ti, return_metadata=True)
        assert not d.any() and not rd.numpy().any()
        np.testing.assert_array_equal(tp, meta["tile_ptr"].numpy())
        assert ids.size == 0
        return
    rd, rtp, rids, rg = _ref(f, to, ti, 3.0, False, 80.0)
    np.testing.assert_array_equal(tp, rtp)
    assert np.abs(d - rd).max() <= 1e-5 * max(np.abs(rd).max(), 1e-30)
    g = oracle.backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tp, ids, **kw)
    for a, b, n in zip(g, rg, ("d_mu", "d_chol_raw", "d_amp")):
        assert np.abs(a - b).max() <= 1e-4 * max(np.abs(b).max(), 1e-30), n
