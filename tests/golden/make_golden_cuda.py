"""Generate golden fixtures from GUASS's own CUDA extension on a GPU.

Runs the reference's compiled cuda_field extension (oracle/_ref, built by
oracle/build_ref.py) on the same seeded cases as make_golden.py and writes
``ref_cuda_<case>.npz`` (inputs, delta, tile_ptr, gaussian_ids in the
reference's stable order, d_mu, d_chol_raw, d_amp).  Run on a GPU box:
    python tests/golden/make_golden_cuda.py --out gpurun_out/golden
then copy the files into tests/golden/.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from guass_b200.synthetic import make_field  # noqa: E402
from oracle import build_ref  # noqa: E402

sys.path.insert(0, str(HERE))
from make_golden import CASES  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE))
    a = ap.parse_args()
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    ext = build_ref.load()
    for name, (out_f, in_f, k, to, ti, sigma, norm, clamp, kw) in CASES.items():
        f = make_field(out_f, in_f, k, seed=0, **kw)
        d = f.to("cuda")
        delta, tp, ids = ext.gaussian_field_forward(d.row_coords, d.col_coords, d.mu, d.chol_raw, d.amp, to, ti,
                                                    sigma, norm, clamp)
        grads = ext.gaussian_field_backward(d.grad, d.row_coords, d.col_coords, d.mu, d.chol_raw, d.amp, tp, ids,
                                            to, ti, sigma, norm, clamp)
        np.savez_compressed(
            out / f"ref_cuda_{name}.npz", out_features=out_f, in_features=in_f, tile_out=to, tile_in=ti,
            sigma=sigma, normalize=int(norm), clamp_quad=np.nan if clamp is None else clamp,
            row_coords=f.row_coords.numpy(), col_coords=f.col_coords.numpy(), mu=f.mu.numpy(),
            chol_raw=f.chol_raw.numpy(), amp=f.amp.numpy(), grad=f.grad.numpy(), delta=delta.cpu().numpy(),
            tile_ptr=tp.cpu().numpy(), gaussian_ids=ids.cpu().numpy(), d_mu=grads[0].cpu().numpy(),
            d_chol_raw=grads[1].cpu().numpy(), d_amp=grads[2].cpu().numpy())
        print(name, "P", ids.numel())


if __name__ == "__main__":
    main()
