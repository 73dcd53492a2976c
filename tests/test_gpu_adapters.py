"""Whole-model adapter binding (guass_b200.adapters) on the CUDA FieldBatch.

Three adapter modules (one with adapter_scale 0.5) render through one batch;
each module's delta must match the CPU oracle for that field, and the
gradients that autograd leaves on mu_raw / chol_raw / amp must match the
exact fp64 gradients of the same field under the condition-aware bound of
tests/gpu_helpers.py (d_mu read back through tanh' = 1 - mu^2).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from torch import nn
from dataclasses import dataclass

import oracle
from guass_b200 import synthetic
from guass_b200.adapters import BatchedAdapters
from gpu_helpers import ATOL, RTOL, assert_grads_exact_within, exact_grads

pytestmark = pytest.mark.gpu


@dataclass
class _Cfg:
    tile_out: int = 32
    tile_in: int = 32
    sigma_multiplier: float = 3.0
    normalize_gaussian: bool = False
    adapter_scale: float = 1.0


class _Adapter(nn.Module):
    def __init__(self, out_f, in_f, k, seed, scale=1.0):
        super().__init__()
        f = synthetic.make_field(out_f, in_f, k, seed=seed, log_scale_mean=math.log(0.06))
        self.field = f
        self.out_features, self.in_features = out_f, in_f
        self.mu_raw = nn.Parameter(torch.atanh(f.mu.clamp(-0.999, 0.999)).cuda())
        self.chol_raw = nn.Parameter(f.chol_raw.clone().cuda())
        self.amp = nn.Parameter(f.amp.clone().cuda())
        self.weight = nn.Parameter(torch.randn(out_f, in_f, device="cuda"))
        self.adapter_config = _Cfg(adapter_scale=scale)
        self.bias = None

    def compute_delta_weight(self):
        raise AssertionError("the binding must replace this")


def _modules():
    return {"q": _Adapter(320, 320, 64, 1), "k": _Adapter(320, 768, 48, 2, scale=0.5),
            "o": _Adapter(130, 70, 9, 3)}


def test_batched_adapters_match_oracle_per_field():
    mods = _modules()
    bank = BatchedAdapters(mods, out_dtype=torch.float32)
    bank.install()
    deltas = bank.render()
    gen = torch.Generator().manual_seed(7)
    grads = [torch.randn(m.out_features, m.in_features, generator=gen) for m in mods.values()]
    loss = sum((m.compute_delta_weight() * g.cuda()).sum() for m, g in zip(mods.values(), grads))
    loss.backward()
    torch.cuda.synchronize()
    assert bank.batch.device_flags() == 0
    for (name, m), d, g in zip(mods.items(), deltas, grads):
        s = m.adapter_config.adapter_scale
        mu = torch.tanh(m.mu_raw.detach()).cpu()  # the values the batch rendered
        f = synthetic.FieldInputs(m.out_features, m.in_features, m.field.row_coords, m.field.col_coords, mu,
                                  m.chol_raw.detach().cpu(), m.amp.detach().cpu(), (g * s).reshape(-1), name=name)
        want, tp, ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp)
        np.testing.assert_allclose(d.detach().cpu().numpy().reshape(-1) / s, want, rtol=RTOL, atol=ATOL)
        d_mu = (m.mu_raw.grad / (1 - torch.tanh(m.mu_raw.detach()).square())).cpu().numpy()
        assert_grads_exact_within([d_mu, m.chol_raw.grad.cpu().numpy(), m.amp.grad.cpu().numpy()],
                                  exact_grads(f, tp, ids), label=f"adapters:{name}")


def test_freeze_and_merge_on_gpu():
    mods = _modules()
    bank = BatchedAdapters(mods, out_dtype=torch.float32)
    bank.install()
    with torch.no_grad():
        live = [d.clone() for d in bank.render()]
        frozen = bank.freeze()
        assert all(torch.equal(a, b) for a, b in zip(live, frozen))
        assert all(m.compute_delta_weight() is d for m, d in zip(mods.values(), frozen))
        bank.unfreeze()
        w0 = [m.weight.detach().clone() for m in mods.values()]
        bank.merge_into_weights()
        for m, w, d in zip(mods.values(), w0, live):
            assert torch.equal(m.weight, w + d)
            assert not m.compute_delta_weight().any()
        bank.unmerge_weights()
        for m, w in zip(mods.values(), w0):
            torch.testing.assert_close(m.weight, w, rtol=0, atol=1e-6)


def test_checkpoint_fields_render_like_the_modules():
    from guass_b200.adapters import CheckpointFields, adapter_state_dict

    mods = {"q": _Adapter(320, 320, 64, 1, scale=0.5), "k": _Adapter(320, 768, 48, 2, scale=0.5)}
    payload = {"format": "gaussian-peft-adapter", "metadata": {"adapter_config": {"adapter_scale": 0.5}},
               "adapters": adapter_state_dict(mods)}
    with torch.no_grad():
        want = [d.clone() for d in BatchedAdapters(mods, out_dtype=torch.float32).render()]
    cf = CheckpointFields(payload, device="cuda", out_dtype=torch.float32)
    got = cf.render()
    assert cf.batch.device_flags() == 0
    for (name, m), w in zip(mods.items(), want):
        assert torch.equal(got[name], w)  # out_scale in the kernel == fp32 multiply after it


def test_trace_events_cover_the_autograd_backward():
    """gf_trace_events is process-wide: the batched render's backward, which
    autograd runs on its own thread, records its four events after the
    forward's three."""
    import ctypes

    from guass_b200 import _lib

    mods = _modules()
    bank = BatchedAdapters(mods, out_dtype=torch.float32, track_metadata=False)
    bank.install()
    L = _lib.lib()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    for e in evs:
        e.record()
    torch.cuda.synchronize()
    handles = (ctypes.c_void_p * 7)(*[e.cuda_event for e in evs])
    _lib.check(L.gf_trace_events(handles, 7))
    try:
        loss = sum((d.float() ** 2).sum() for d in bank.render())
        loss.backward()
        torch.cuda.synchronize()
        assert L.gf_trace_count() == 7
    finally:
        _lib.check(L.gf_trace_events(None, 0))
    times = [evs[k].elapsed_time(evs[k + 1]) for k in range(6)]
    assert all(t >= 0.0 for t in times)
