"""Exact properties of the CUDA path at full BASELINE size (see
tests/property_checks.py for why they hold bit for bit): the whole SD1.5-UNet
batch (cfg3, 128 fields, 93.5 M delta elements) and the 1280x1280 K=1024
field (cfg2)."""
from __future__ import annotations

import pytest
import torch

from guass_b200 import synthetic
from guass_b200.batched import FieldBatch, pack_fields
from property_checks import (check_amp_linearity, check_batch_equals_single, check_binning_invariants,
                             check_grad_linearity)

pytestmark = pytest.mark.gpu


def _bound(shapes):
    # the exact upper bound on pairs: every Gaussian in every tile
    return sum(k * ((o + 31) // 32) * ((i + 31) // 32) for o, i, k in shapes)


def _factory(out_dtype=torch.bfloat16):
    return lambda shapes: FieldBatch(shapes, out_dtype=out_dtype, ids_capacity=_bound(shapes))


@pytest.fixture(scope="module")
def unet():
    fields = synthetic.cfg3()
    shapes = [(f.out_features, f.in_features, f.k) for f in fields]
    return shapes, pack_fields(fields, device="cuda")


def test_unet_amp_and_grad_linearity(unet):
    shapes, (mu, chol, amp, grad) = unet
    b = _factory()(shapes)
    check_amp_linearity(b, mu, chol, amp)
    check_grad_linearity(b, mu, chol, amp, grad)
    assert b.device_flags() == 0


def test_unet_batch_equals_single_fields(unet):
    shapes, (mu, chol, amp, grad) = unet
    check_batch_equals_single(_factory(), shapes, mu, chol, amp, grad, pick=[0, 5, 40, 77, 127])


def test_unet_binning_invariants(unet):
    shapes, (mu, chol, amp, grad) = unet
    b = _factory()(shapes)
    b.forward(mu, chol, amp)
    assert b.device_flags() == 0
    base = b.pair_base.cpu().numpy()
    ids = b.ids.cpu().numpy()
    for f, (o, i, k) in enumerate(shapes):
        tp = b.tile_ptr_view(f).cpu().numpy()
        check_binning_invariants(tp, ids[base[f]:base[f + 1]], k, b.num_tiles[f])


def test_cfg2_linearity_fp32():
    f = synthetic.cfg2()
    shapes = [(f.out_features, f.in_features, f.k)]
    mu, chol, amp, grad = pack_fields([f], device="cuda")
    b = _factory(torch.float32)(shapes)
    check_amp_linearity(b, mu, chol, amp)
    check_grad_linearity(b, mu, chol, amp, grad)
