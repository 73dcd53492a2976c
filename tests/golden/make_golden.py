"""Generate golden fixtures from GUASS's own PyTorch path (run where the
reference package is importable; the GPU box does not need it).

For each small seeded case this runs the reference's
``gaussian_peft.kernels.gaussian_field(..., execution_mode="tiled_reference_pytorch")``
(gaussian_peft/kernels/gaussian_field.py:18-97) forward and autograd backward on
the CPU and stores inputs and outputs in ``ref_torch_<case>.npz``:

  inputs   out_features, in_features, tile_out, tile_in, sigma, normalize,
           clamp_quad, row_coords, col_coords, mu, chol_raw, amp, grad
  outputs  delta, tile_ptr, gaussian_ids (per tile in the reference's order),
           d_mu, d_chol_raw, d_amp, and the bounds (tile_r0/r1/c0/c1)

Usage:  python tests/golden/make_golden.py [--reference /root/reference]
"""
from __future__ import annotations

import argparse
import os
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from guass_b200.synthetic import make_field  # noqa: E402

CASES = {
    # name: (out, in, K, tile_out, tile_in, sigma, normalize, clamp, field kwargs)
    "small_default": (96, 160, 24, 32, 32, 3.0, False, 80.0, dict(log_scale_mean=math.log(0.08))),
    "ragged_norm": (70, 45, 10, 16, 8, 2.5, True, 80.0, dict(log_scale_mean=math.log(0.1))),
    "noclamp_wide": (33, 130, 12, 32, 32, 3.0, False, None, dict(log_scale_mean=math.log(0.3), log_scale_std=0.8)),
    "single_gaussian": (64, 64, 1, 32, 32, 3.0, False, 80.0, dict(log_scale_mean=math.log(0.1))),
    "one_row": (1, 40, 5, 32, 32, 3.0, False, 80.0, dict(log_scale_mean=math.log(0.1))),
    "elongated": (64, 96, 16, 32, 32, 3.0, False, 80.0,
                  dict(log_scale_mean=math.log(0.15), elongated_frac=0.5, elongation=(5.0, 20.0))),
}


def run_case(name, spec, seed=0):
    from gaussian_peft.kernels.covariance import activate_cholesky
    from gaussian_peft.kernels.bounds import compute_gaussian_tile_bounds
    from gaussian_peft.kernels.gaussian_field import gaussian_field

    out_f, in_f, k, to, ti, sigma, norm, clamp, kw = spec
    f = make_field(out_f, in_f, k, seed=seed, **kw)
    mu = f.mu.clone().requires_grad_(True)
    chol_raw = f.chol_raw.clone().requires_grad_(True)
    amp = f.amp.clone().requires_grad_(True)
    chol = activate_cholesky(chol_raw, eps=1e-5)
    coords = torch.zeros(1, 2)
    delta, meta = gaussian_field(coords, mu, chol, amp, normalize=norm, clamp_quad=clamp,
                                 execution_mode="tiled_reference_pytorch", row_coords=f.row_coords,
                                 col_coords=f.col_coords, tile_out=to, tile_in=ti, sigma_multiplier=sigma,
                                 return_metadata=True)
    delta.backward(f.grad)
    bounds = compute_gaussian_tile_bounds(mu.detach(), chol.detach(), out_f, in_f, to, ti, sigma)
    return dict(
        out_features=out_f, in_features=in_f, tile_out=to, tile_in=ti, sigma=sigma, normalize=int(norm),
        clamp_quad=np.nan if clamp is None else clamp,
        row_coords=f.row_coords.numpy(), col_coords=f.col_coords.numpy(), mu=f.mu.numpy(),
        chol_raw=f.chol_raw.numpy(), amp=f.amp.numpy(), grad=f.grad.numpy(),
        delta=delta.detach().numpy(), tile_ptr=meta["tile_ptr"].numpy(), gaussian_ids=meta["gaussian_ids"].numpy(),
        d_mu=mu.grad.numpy(), d_chol_raw=chol_raw.grad.numpy(), d_amp=amp.grad.numpy(),
        tile_r0=bounds.tile_r0.numpy(), tile_r1=bounds.tile_r1.numpy(), tile_c0=bounds.tile_c0.numpy(),
        tile_c1=bounds.tile_c1.numpy(),
    )


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GUASS_REFERENCE_ROOT", "/root/reference"))
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    torch.set_num_threads(1)
    for name, spec in CASES.items():
        data = run_case(name, spec)
        path = HERE / f"ref_torch_{name}.npz"
        np.savez_compressed(path, **data)
        print(f"{path.name}: P={data['gaussian_ids'].size} |delta|max={np.abs(data['delta']).max():.3e}")


if __name__ == "__main__":
    main()
