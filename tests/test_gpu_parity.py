"""CUDA product path vs the CPU oracle, through the C ABI (via the drop-in shim).

Binning (tile_ptr, gaussian_ids_sorted) must be bit-exact; fp32 delta within
1e-5 rel / 1e-7 abs per element (the oracle's host expf differs from CUDA's
by an ulp or two); gradients within 1e-5 of their channel scale + 1e-7.
"""
from __future__ import annotations


import numpy as np
import pytest
import torch

from guass_b200 import synthetic as S
from gpu_helpers import (ATOL, RTOL, assert_grads_exact_within, exact_grads, random_field,
                         run_ext, run_oracle)

pytestmark = pytest.mark.gpu


def _check(f, label="", **kw):
    d_g, tp_g, ids_g, gr_g = run_ext(f, **kw)
    d_o, tp_o, ids_o, _ = run_oracle(f, **kw)
    np.testing.assert_array_equal(tp_g, tp_o)
    np.testing.assert_array_equal(ids_g, ids_o)
    np.testing.assert_allclose(d_g, d_o, rtol=RTOL, atol=ATOL)
    keys = ("tile_out", "tile_in", "sigma", "normalize", "clamp", "grad")
    assert_grads_exact_within(gr_g, exact_grads(f, tp_o, ids_o, **{k: v for k, v in kw.items() if k in keys}),
                              label=label or f.name)


@pytest.mark.parametrize("cfg", ["cfg0", "cfg1", "cfg2"])
def test_benchmark_configs(cfg):
    _check(S.CONFIGS[cfg](), label=f"gpu_vs_exact:{cfg}")


@pytest.mark.parametrize("normalize,clamp", [(True, 80.0), (False, None), (True, None), (False, 8.0)])
def test_normalize_and_clamp_variants(normalize, clamp):
    _check(random_field(200, 300, 80, seed=11, mean_scale=0.08), normalize=normalize, clamp=clamp)


@pytest.mark.parametrize("shape,tiles", [
    ((70, 45), (16, 8)),     # ragged edges, small tiles
    ((33, 130), (32, 32)),   # partial tile rows
    ((1, 40), (32, 32)),     # single row
    ((40, 1), (32, 32)),     # single column
    ((100, 200), (64, 64)),  # tiles larger than one 32x32 sub-block
    ((90, 77), (7, 13)),     # odd tile sizes
    ((64, 300), (8, 96)),    # wide tiles, 3 column sub-blocks
    ((1, 1), (32, 32)),      # one element
    ((3, 20), (64, 64)),     # one tile larger than the whole field
])
def test_tile_shapes(shape, tiles):
    f = random_field(shape[0], shape[1], 30, seed=5, mean_scale=0.1)
    _check(f, tile_out=tiles[0], tile_in=tiles[1])


def test_sigma_multiplier():
    _check(random_field(160, 160, 40, seed=2, mean_scale=0.06), sigma=1.7)


def test_single_and_empty_field():
    _check(random_field(64, 64, 1, seed=1, mean_scale=0.1))
    f = random_field(64, 96, 1, seed=1)
    f.mu, f.chol_raw, f.amp = f.mu[:0], f.chol_raw[:0], f.amp[:0]
    d_g, tp_g, ids_g, gr_g = run_ext(f)
    assert ids_g.size == 0 and np.all(tp_g == 0) and np.all(d_g == 0)
    assert all(g.shape[0] == 0 for g in gr_g)


def test_many_gaussians_per_tile():
    # > 256 candidates per tile: several compaction chunks in one tile
    f = random_field(96, 96, 1200, seed=4, mean_scale=0.2, spread=0.2)
    _check(f)


def test_gaussians_far_outside_and_huge():
    f = random_field(128, 256, 50, seed=9, mean_scale=0.05)
    f.mu[:10] = f.mu[:10] * 4.0                      # centres far outside [-1, 1]
    f.chol_raw[10:15, 0] = 3.0                        # very wide
    f.chol_raw[10:15, 2] = 3.0
    f.chol_raw[15:20, 0] = -12.0                      # tiny (det at the floor)
    f.chol_raw[15:20, 2] = -12.0
    _check(f)


def test_zero_gradient_elements_are_skipped():
    f = random_field(96, 128, 40, seed=6, mean_scale=0.08)
    g = f.grad.clone()
    g[::3] = 0.0
    _check(f, grad=g)


def test_bf16_output_matches_rne_cast():
    from guass_b200.cuda_field import load_extension

    f = S.cfg1().to("cuda")
    ext = load_extension()
    d32, tp, ids = ext.gaussian_field_forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, 32, 32, 3.0,
                                              False, 80.0)
    d16, tp16, ids16 = ext.forward_into(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, 32, 32, 3.0, False,
                                        80.0, out_dtype=torch.bfloat16)
    assert torch.equal(tp, tp16) and torch.equal(ids, ids16)
    # reference: fp32 delta then .to(bf16) (gaussian_linear.py:236), round-to-nearest-even
    assert torch.equal(d16, d32.to(torch.bfloat16))
    rel = ((d16.float() - d32).abs() <= 1e-2 * d32.abs() + 1e-30).float().mean()
    assert float(rel) == 1.0


def test_out_scale_matches_scaled_fp32():
    from guass_b200.cuda_field import load_extension

    f = S.cfg0().to("cuda")
    ext = load_extension()
    d, _, _ = ext.forward_into(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, 32, 32, 3.0, False, 80.0)
    ds, _, _ = ext.forward_into(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, 32, 32, 3.0, False, 80.0,
                                out_scale=0.37)
    assert torch.equal(ds, d * 0.37)


def test_bf16_gradient_input():
    f = S.cfg1()
    g16 = f.grad.to(torch.bfloat16)
    d_g, tp_g, ids_g, gr_g = run_ext(f, grad=g16)
    assert_grads_exact_within(gr_g, exact_grads(f, tp_g, ids_g, grad=g16.float()), label="bf16_grad")


def test_backward_is_bitwise_deterministic():
    f = S.cfg2()
    a = run_ext(f)
    b = run_ext(f)
    for x, y in zip(a[3], b[3]):
        assert np.array_equal(x, y)
    assert np.array_equal(a[0], b[0])


def test_int32_saved_indices_accepted():
    from guass_b200.cuda_field import load_extension

    f = S.cfg0().to("cuda")
    ext = load_extension()
    delta, tp, ids = ext.gaussian_field_forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, 32, 32, 3.0,
                                                False, 80.0)
    g64 = ext.gaussian_field_backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tp, ids, 32, 32,
                                      3.0, False, 80.0)
    g32 = ext.gaussian_field_backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp,
                                      tp.to(torch.int32), ids.to(torch.int32), 32, 32, 3.0, False, 80.0)
    for x, y in zip(g64, g32):
        assert torch.equal(x, y)


def test_inconsistent_saved_state_is_reported(monkeypatch):
    """Device-side saved-state checks (field_impl.cu:86-108 does these on the
    host): a foreign id is skipped by the kernel and reported, not read."""
    import guass_b200.cuda_field._ext as E

    monkeypatch.setattr(E, "_VALIDATE", True)
    f = S.cfg0().to("cuda")
    ext = E.GaussianFieldExtension()
    delta, tp, ids = ext.gaussian_field_forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, 32, 32, 3.0,
                                                False, 80.0)
    bad = ids.clone()
    bad[3] = 10_000  # out of range
    with pytest.raises(RuntimeError, match="do not match"):
        ext.gaussian_field_backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tp, bad, 32, 32,
                                    3.0, False, 80.0)
    shuffled = ids.clone()
    seg = shuffled[int(tp[5]):int(tp[6])]
    if seg.numel() >= 2:
        shuffled[int(tp[5]):int(tp[6])] = seg.flip(0)
        with pytest.raises(RuntimeError, match="do not match"):
            ext.gaussian_field_backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tp, shuffled,
                                        32, 32, 3.0, False, 80.0)
    # a clean call afterwards works
    ext.gaussian_field_backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tp, ids, 32, 32, 3.0,
                                False, 80.0)


def test_autograd_runtime_matches_extension():
    from guass_b200.cuda_field import gaussian_field_train

    f = S.cfg1().to("cuda")
    mu = f.mu.clone().requires_grad_(True)
    chol = f.chol_raw.clone().requires_grad_(True)
    amp = f.amp.clone().requires_grad_(True)
    delta = gaussian_field_train(row_coords=f.row_coords, col_coords=f.col_coords, mu=mu, chol_raw=chol, amp=amp,
                                 tile_out=32, tile_in=32, sigma_multiplier=3.0)
    delta.backward(f.grad)
    d_g, _, _, gr = run_ext(f)
    assert np.array_equal(delta.detach().cpu().numpy(), d_g)
    for p, want in zip((mu, chol, amp), gr):
        assert np.array_equal(p.grad.cpu().numpy(), want)
