"""Fused-weight epilogue of the forward (gf_field.base_weight) on the B200.

With a base weight W0 the forward stores out(float(W0) + out_scale * value)
with one rounding.  The value is the same fp32 number the plain fp32 render
stores, so every case here is bit-exact against ``(W0.float() + D32).to(out)``:
bf16 and fp32 outputs, widths that take the 128-bit and the scalar store
paths, the 32x32 fast kernels and the generic kernels (16x16 tiles), a
multi-field batch, and the in-place form (base_weight == delta).  The
backward does not read the base, so its gradients must not change.
"""
from __future__ import annotations

import pytest
import torch

from guass_b200 import synthetic
from guass_b200.batched import FieldBatch, pack_fields

pytestmark = pytest.mark.gpu

SCALE = 0.75


def _fields():
    # 320x768: vector stores; 130x70: ragged tiles and scalar stores (70 % 8 != 0)
    return [synthetic.make_field(320, 768, 256, seed=4), synthetic.make_field(130, 70, 40, seed=5),
            synthetic.make_field(64, 96, 16, seed=6)]


@pytest.mark.parametrize("tile", [32, 16])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_fused_weight_is_base_plus_scaled_value(tile, out_dtype):
    fields = _fields()
    shapes = [(f.out_features, f.in_features, f.k) for f in fields]
    mu, chol, amp, grad = pack_fields(fields, device="cuda")
    cap = sum(k * -(-o // tile) * -(-i // tile) for o, i, k in shapes)  # every Gaussian in every tile
    kw = dict(tile_out=tile, tile_in=tile, out_scale=SCALE, ids_capacity=cap)
    d32 = FieldBatch(shapes, out_dtype=torch.float32, **kw).forward(mu, chol, amp).clone()
    n = d32.numel()
    w0 = torch.randn(n, generator=torch.Generator().manual_seed(9)).to("cuda", out_dtype)
    want = (w0.float() + d32).to(out_dtype)
    w0_copy = w0.clone()

    b = FieldBatch(shapes, out_dtype=out_dtype, base_weight=w0, **kw)
    got = b.forward(mu, chol, amp)
    assert b.device_flags() == 0
    assert torch.equal(got, want)
    assert torch.equal(w0, w0_copy)  # the base is only read

    # in place: the output buffer holds W0 before the render
    ip = FieldBatch(shapes, out_dtype=out_dtype, **kw)
    ip.delta.copy_(w0)
    ip.set_base_weight(ip.delta)
    assert torch.equal(ip.forward(mu, chol, amp), want)

    # the backward ignores the base
    g = grad.to(torch.float32)
    plain = FieldBatch(shapes, out_dtype=out_dtype, **kw)
    plain.forward(mu, chol, amp)
    want_g = [t.clone() for t in plain.backward(g, mu, chol, amp)]
    got_g = b.backward(g, mu, chol, amp)
    for a, w in zip(got_g, want_g):
        assert torch.equal(a, w)


def test_base_weight_checked():
    shapes = [(64, 64, 8)]
    with pytest.raises(ValueError, match="base_weight"):
        FieldBatch(shapes, out_dtype=torch.bfloat16, base_weight=torch.zeros(64 * 64, device="cuda"))
    with pytest.raises(ValueError, match="base_weight"):
        FieldBatch(shapes, out_dtype=torch.float32, base_weight=torch.zeros(64 * 63, device="cuda"))
