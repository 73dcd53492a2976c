"""The bounds-checked debug build (libgfield_check.so, -DGF_CHECK) on the B200.

The same cases run through the checked library (in a subprocess, selected
with GUASS_B200_LIB) and through the release library (here): the checked run
must record no GF_FLAG_BOUNDS (or any other flag), the deltas must be
bit-identical and the gradients equal to a few ulp -- the checks only observe.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def run_cases() -> dict:
    from guass_b200 import synthetic
    from guass_b200.batched import FieldBatch, pack_fields

    out = {}
    cases = {
        "cfg0_f32": ([synthetic.cfg0()], dict(out_dtype=torch.float32)),
        "ragged_generic": ([synthetic.make_field(130, 70, 40, seed=5), synthetic.make_field(33, 47, 9, seed=6)],
                           dict(out_dtype=torch.float32, tile_out=16, tile_in=8)),
        "bf16_base": ([synthetic.make_field(320, 768, 256, seed=4)], dict(out_dtype=torch.bfloat16)),
    }
    for name, (fields, kw) in cases.items():
        shapes = [(f.out_features, f.in_features, f.k) for f in fields]
        mu, chol, amp, grad = pack_fields(fields, device="cuda")
        cap = sum(k * -(-o // kw.get("tile_out", 32)) * -(-i // kw.get("tile_in", 32)) for o, i, k in shapes)
        b = FieldBatch(shapes, ids_capacity=cap, **kw)
        if name == "bf16_base":
            b.set_base_weight(torch.linspace(-1, 1, b.numel(), device="cuda").to(torch.bfloat16))
        d = b.forward(mu, chol, amp).float().cpu().numpy()
        g = [t.cpu().numpy() for t in b.backward(grad, mu, chol, amp)]
        out[name + ".delta"] = d
        for n, t in zip(("d_mu", "d_chol_raw", "d_amp"), g):
            out[f"{name}.{n}"] = t
        out[name + ".flags"] = np.array([b.device_flags()])
    return out


def test_checked_build_agrees_and_flags_nothing(tmp_path):
    from guass_b200 import _build

    check_lib = _build.LIB_CHECK
    if not check_lib.exists():
        pytest.fail(f"{check_lib} is missing: build it with python -m guass_b200._build")
    path = tmp_path / "checked.npz"
    env = dict(os.environ, GUASS_B200_LIB=str(check_lib),
               PYTHONPATH=os.pathsep.join([str(ROOT), str(ROOT / "tests"), os.environ.get("PYTHONPATH", "")]))
    code = ("import numpy as np, sys, test_gpu_check_build as t; "
            f"np.savez({str(path)!r}, **t.run_cases())")
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    checked = dict(np.load(path))
    release = run_cases()
    assert set(checked) == set(release)
    for key in sorted(checked):
        if key.endswith(".flags"):
            assert checked[key][0] == 0, f"{key}: checked build recorded flags {checked[key][0]:#x}"
            assert release[key][0] == 0
        elif key.endswith(".delta"):
            assert np.array_equal(checked[key], release[key]), key  # explicit-rounding arithmetic: bitwise
        else:
            # gradients: the same operations, but the compiler may contract a plain a*b+c differently
            # around the added branches; held to a few ulp of the array's scale
            scale = max(float(np.abs(release[key]).max()), 1e-30)
            assert float(np.abs(checked[key] - release[key]).max()) <= 1e-6 * scale, key
