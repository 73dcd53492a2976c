"""Optional backward basis from the base-2 hardware approximation
(GF_CFG_BWD_EXP2) on the B200: the forward's delta is unchanged bit for bit and
the gradients stay within the condition-aware bound of tests/gpu_helpers.py
that the expf backward (and the reference's own extension) is held to."""
from __future__ import annotations

import pytest
import torch

from guass_b200 import synthetic as S
from gpu_helpers import assert_grads_exact_within, exact_grads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", ["cfg0", "cfg1", "cfg2"])
def test_backward_exp2_basis_within_tolerance(cfg):
    """GF_CFG_BWD_EXP2 (backward basis from ex2.approx): delta unchanged bit
    for bit, gradients held to the same condition-aware bound as expf."""
    from guass_b200.batched import FieldBatch, pack_fields

    f = S.CONFIGS[cfg]()
    shapes = [(f.out_features, f.in_features, f.k)]
    mu, chol, amp, grad = pack_fields([f], device="cuda")
    cap = f.k * -(-f.out_features // 32) * -(-f.in_features // 32)
    ref = FieldBatch(shapes, out_dtype=torch.float32, ids_capacity=cap)
    fast = FieldBatch(shapes, out_dtype=torch.float32, ids_capacity=cap, bwd_exp2=True)
    d_ref = ref.forward(mu, chol, amp).clone()
    d_fast = fast.forward(mu, chol, amp).clone()
    assert torch.equal(d_ref, d_fast)
    got = [t.cpu().numpy() for t in fast.backward(grad, mu, chol, amp)]
    assert fast.device_flags() == 0
    tp = fast.tile_ptr_view(0).cpu().numpy()
    ids = fast.ids[:int(tp[-1])].cpu().numpy()
    assert_grads_exact_within(got, exact_grads(f, tp, ids), label=f"bwd_exp2:{cfg}")


@pytest.mark.parametrize("normalize,clamp", [(True, 80.0), (False, None), (True, None), (False, 8.0)])
def test_backward_exp2_basis_normalize_and_clamp_variants(normalize, clamp):
    from guass_b200.batched import FieldBatch, pack_fields
    from gpu_helpers import random_field

    f = random_field(200, 300, 80, seed=11, mean_scale=0.08)
    shapes = [(f.out_features, f.in_features, f.k)]
    mu, chol, amp, grad = pack_fields([f], device="cuda")
    cap = f.k * -(-f.out_features // 32) * -(-f.in_features // 32)
    kw = dict(out_dtype=torch.float32, ids_capacity=cap, normalize=normalize, clamp_quad=clamp)
    ref = FieldBatch(shapes, **kw)
    fast = FieldBatch(shapes, bwd_exp2=True, **kw)
    assert torch.equal(ref.forward(mu, chol, amp).clone(), fast.forward(mu, chol, amp).clone())
    got = [t.cpu().numpy() for t in fast.backward(grad, mu, chol, amp)]
    assert fast.device_flags() == 0
    tp = fast.tile_ptr_view(0).cpu().numpy()
    ids = fast.ids[:int(tp[-1])].cpu().numpy()
    assert_grads_exact_within(got, exact_grads(f, tp, ids, normalize=normalize, clamp=clamp),
                              label=f"bwd_exp2:norm={normalize},clamp={clamp}")
