"""The exact properties of tests/property_checks.py on the CPU oracle.

This validates the checks themselves (and the oracle) on small fields; the GPU
test applies the same checks to the CUDA path at full size."""
from __future__ import annotations

import math

import numpy as np
import torch

import oracle
from guass_b200 import synthetic
from property_checks import (check_amp_linearity, check_batch_equals_single, check_binning_invariants,
                             check_grad_linearity)
from oracle_batch import OracleBatch

KW = dict(tile_out=32, tile_in=32, sigma_multiplier=3.0, normalize=False, clamp_quad=80.0)


def _fields():
    return [synthetic.make_field(o, i, k, seed=s, log_scale_mean=math.log(0.06))
            for s, (o, i, k) in enumerate([(64, 96, 20), (40, 70, 9), (96, 64, 30)])]


def _packed(fields):
    return (torch.cat([f.mu for f in fields]), torch.cat([f.chol_raw for f in fields]),
            torch.cat([f.amp for f in fields]), torch.cat([f.grad for f in fields]))


def test_linearity_on_oracle():
    fields = _fields()
    shapes = [(f.out_features, f.in_features, f.k) for f in fields]
    mu, chol, amp, grad = _packed(fields)
    check_amp_linearity(OracleBatch(shapes, **KW), mu, chol, amp)
    check_grad_linearity(OracleBatch(shapes, **KW), mu, chol, amp, grad)


def test_batch_equals_single_on_oracle():
    fields = _fields()
    shapes = [(f.out_features, f.in_features, f.k) for f in fields]
    check_batch_equals_single(lambda sh: OracleBatch(sh, **KW), shapes, *_packed(fields), pick=[0, 2])


def test_binning_invariants_on_oracle():
    for f in _fields() + [synthetic.cfg2()]:
        _, tp, ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp)
        nt = ((f.out_features + 31) // 32) * ((f.in_features + 31) // 32)
        check_binning_invariants(tp, ids, f.k, nt)


def test_checks_detect_a_broken_render():
    """A render that is off by one ulp somewhere must fail the linearity check."""
    fields = _fields()
    shapes = [(f.out_features, f.in_features, f.k) for f in fields]
    mu, chol, amp, _ = _packed(fields)

    class Broken(OracleBatch):
        def forward(self, m, c, a):
            d = super().forward(m, c, a)
            if float(a.abs().max()) > float(amp.abs().max()):  # the doubled call
                d[7] = np.nextafter(np.float32(d[7]), np.float32(1)).item()
            return d

    try:
        check_amp_linearity(Broken(shapes, **KW), mu, chol, amp)
    except AssertionError:
        return
    raise AssertionError("the linearity check did not notice a one-ulp change")


from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402


@settings(max_examples=40, deadline=None)
@given(out_f=st.integers(1, 90), in_f=st.integers(1, 90), k=st.integers(0, 24),
       tiles=st.sampled_from([(32, 32), (8, 8), (16, 7), (13, 64), (64, 64)]),
       sigma=st.sampled_from([1.0, 2.0, 3.0, 4.5]), scale=st.sampled_from([0.02, 0.1, 0.4]),
       seed=st.integers(0, 2 ** 16))
def test_binning_equals_brute_force_from_boxes(out_f, in_f, k, tiles, sigma, scale, seed):
    """The oracle's counting-sort binning (forward.cu:211-252 restated) equals a
    brute-force construction from its own per-Gaussian tile boxes: tile t lists
    every Gaussian whose box contains t, in ascending id order."""
    to, ti = tiles
    f = synthetic.make_field(out_f, in_f, k, seed=seed, log_scale_mean=math.log(scale), elongated_frac=0.3)
    geo = oracle.preprocess(out_f, in_f, f.mu, f.chol_raw, tile_out=to, tile_in=ti, sigma_multiplier=sigma)
    _, tp, ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tile_out=to, tile_in=ti,
                                sigma_multiplier=sigma)
    ntr, ntc = -(-out_f // to), -(-in_f // ti)
    assert tp.size == ntr * ntc + 1
    for t in range(ntr * ntc):
        tr, tc = divmod(t, ntc)
        want = [g for g in range(k) if geo["r0"][g] <= tr <= geo["r1"][g] and geo["c0"][g] <= tc <= geo["c1"][g]]
        assert list(ids[tp[t]:tp[t + 1]]) == want, t
    # each Gaussian appears once per tile of its box (tiles_touched, forward.cu:203-208)
    assert np.array_equal(np.bincount(ids.astype(np.int64), minlength=k), geo["tiles_touched"])
