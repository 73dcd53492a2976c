"""The CPU oracle against golden vectors made by GUASS's own code.

``ref_torch_*.npz`` come from the reference's PyTorch path
(gaussian_peft/kernels/gaussian_field.py, tiled_reference_pytorch) run by
tests/golden/make_golden.py.  That path bins with an unstable argsort
(gaussian_peft/kernels/tile_index.py:86), so ids are compared per tile as sets;
bounds and tile_ptr must match exactly.  ``ref_cuda_*.npz`` (when present) come
from the reference's CUDA extension on a B200 (tests/golden/make_golden_cuda.py)
and pin the stable order bit for bit.
"""
from __future__ import annotations

import glob
from pathlib import Path

import numpy as np
import pytest

import oracle
from ref_defects import reference_undefined_tiles, tile_mask_to_elements

GOLDEN = Path(__file__).resolve().parent / "golden"
TORCH_CASES = sorted(glob.glob(str(GOLDEN / "ref_torch_*.npz")))
CUDA_CASES = sorted(glob.glob(str(GOLDEN / "ref_cuda_*.npz")))

# The torch path computes Sigma^-1 with torch.linalg.inv and det with
# torch.linalg.det (gaussian_peft/kernels/gaussian_core.py:43-44), not the
# analytic formulas, so it agrees with the CUDA arithmetic to ~1e-6 of scale.
TORCH_RTOL_OF_MAX = 1e-5


def _kw(d):
    clamp = None if np.isnan(d["clamp_quad"]) else float(d["clamp_quad"])
    return dict(tile_out=int(d["tile_out"]), tile_in=int(d["tile_in"]), sigma_multiplier=float(d["sigma"]),
                normalize=bool(d["normalize"]), clamp_quad=clamp)


def _rel_of_max(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def test_golden_fixtures_present():
    assert len(TORCH_CASES) >= 6


@pytest.mark.parametrize("path", TORCH_CASES, ids=lambda p: Path(p).stem)
def test_oracle_matches_reference_torch_path(path):
    d = np.load(path)
    kw = _kw(d)
    out_f, in_f = int(d["out_features"]), int(d["in_features"])
    geo = oracle.preprocess(out_f, in_f, d["mu"], d["chol_raw"], kw["tile_out"], kw["tile_in"], kw["sigma_multiplier"])
    for a, b in (("r0", "tile_r0"), ("r1", "tile_r1"), ("c0", "tile_c0"), ("c1", "tile_c1")):
        np.testing.assert_array_equal(geo[a], d[b])
    delta, tile_ptr, ids = oracle.forward(d["row_coords"], d["col_coords"], d["mu"], d["chol_raw"], d["amp"], **kw)
    np.testing.assert_array_equal(tile_ptr, d["tile_ptr"])
    for t in range(tile_ptr.size - 1):
        seg = ids[tile_ptr[t]:tile_ptr[t + 1]]
        assert np.all(np.diff(seg) > 0), "oracle ids must ascend inside a tile (stable sort)"
        assert sorted(seg) == sorted(d["gaussian_ids"][tile_ptr[t]:tile_ptr[t + 1]])
    assert _rel_of_max(delta, d["delta"]) < TORCH_RTOL_OF_MAX
    grads = oracle.backward(d["grad"], d["row_coords"], d["col_coords"], d["mu"], d["chol_raw"], d["amp"], tile_ptr,
                            ids, **kw)
    for g, name in zip(grads, ("d_mu", "d_chol_raw", "d_amp")):
        assert _rel_of_max(g, d[name]) < TORCH_RTOL_OF_MAX, name


@pytest.mark.parametrize("path", CUDA_CASES, ids=lambda p: Path(p).stem)
def test_oracle_matches_reference_cuda_extension(path):
    d = np.load(path)
    kw = _kw(d)
    delta, tile_ptr, ids = oracle.forward(d["row_coords"], d["col_coords"], d["mu"], d["chol_raw"], d["amp"], **kw)
    np.testing.assert_array_equal(tile_ptr, d["tile_ptr"])
    np.testing.assert_array_equal(ids, d["gaussian_ids"])
    # host libm expf vs CUDA expf: a few ulp per term; tiles where the
    # reference reads uninitialised shared memory are excluded
    out_f, in_f, to, ti = (int(d[k]) for k in ("out_features", "in_features", "tile_out", "tile_in"))
    defined = ~tile_mask_to_elements(reference_undefined_tiles(out_f, in_f, to, ti, tile_ptr), out_f, in_f, to, ti)
    np.testing.assert_allclose(delta[defined], d["delta"][defined], rtol=1e-5, atol=1e-7)
    grads = oracle.backward(d["grad"], d["row_coords"], d["col_coords"], d["mu"], d["chol_raw"], d["amp"], tile_ptr,
                            ids, **kw)
    for g, name in zip(grads, ("d_mu", "d_chol_raw", "d_amp")):
        assert _rel_of_max(g, d[name]) < 1e-5, name


def test_oracle_empty_field():
    row = np.linspace(-1, 1, 40, dtype=np.float32)
    col = np.linspace(-1, 1, 50, dtype=np.float32)
    delta, tp, ids = oracle.forward(row, col, np.zeros((0, 2)), np.zeros((0, 3)), np.zeros((0, 1)))
    assert ids.size == 0 and np.all(tp == 0) and np.all(delta == 0)


def test_oracle_counting_sort_is_stable_sort():
    rng = np.random.default_rng(3)
    k = 300
    mu = rng.uniform(-1.2, 1.2, (k, 2)).astype(np.float32)
    chol = np.stack([rng.normal(-3, 1, k), rng.normal(0, 0.05, k), rng.normal(-3, 1, k)], 1).astype(np.float32)
    geo = oracle.preprocess(200, 300, mu, chol)
    tp, ids = oracle.bin_pairs(200, 300, geo)
    keys, gids = [], []
    ntc = (300 + 31) // 32
    for g in range(k):  # forward.cu:211-241 emission order
        for tr in range(geo["r0"][g], geo["r1"][g] + 1):
            for tc in range(geo["c0"][g], geo["c1"][g] + 1):
                keys.append(tr * ntc + tc)
                gids.append(g)
    order = np.argsort(np.asarray(keys), kind="stable")
    np.testing.assert_array_equal(ids, np.asarray(gids)[order])
    assert tp[-1] == len(keys)
