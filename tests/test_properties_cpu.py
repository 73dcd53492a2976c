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
from test_adapters import OracleBatch

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
