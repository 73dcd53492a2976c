"""Staged forward (gf_forward_stages) on one B200.

BIN then RENDER equals gf_forward bit for bit; and the schedule the fused
multi-GPU exchange uses -- binning (which, run alone, also writes the
per-tile id lists), then the backward on a second stream (its own workspace)
while the render runs -- gives the same delta and gradients as the plain
sequence.
"""
from __future__ import annotations

import pytest
import torch

from guass_b200 import _lib, synthetic
from guass_b200.batched import FieldBatch, pack_fields

pytestmark = pytest.mark.gpu


def _setup():
    fields = synthetic.cfg3()[:24]
    shapes = [(f.out_features, f.in_features, f.k) for f in fields]
    mu, chol, amp, grad = pack_fields(fields, device="cuda")
    cap = sum(k * -(-o // 32) * -(-i // 32) for o, i, k in shapes)
    return shapes, (mu, chol, amp, grad), cap


def test_stages_equal_the_full_forward():
    shapes, (mu, chol, amp, grad), cap = _setup()
    a = FieldBatch(shapes, ids_capacity=cap)
    b = FieldBatch(shapes, ids_capacity=cap)
    want = a.forward(mu, chol, amp).clone()
    b.forward_stages(mu, chol, amp, _lib.GF_STAGE_BIN)
    b.forward_stages(mu, chol, amp, _lib.GF_STAGE_RENDER)
    assert torch.equal(b.delta, want)
    assert torch.equal(b.tile_ptr, a.tile_ptr) and torch.equal(b.pair_base, a.pair_base)
    assert a.device_flags() == 0 and b.device_flags() == 0


def test_backward_overlapping_the_render_matches_the_sequence():
    shapes, (mu, chol, amp, grad), cap = _setup()
    seq = FieldBatch(shapes, ids_capacity=cap)
    seq.forward(mu, chol, amp)
    want_delta = seq.delta.clone()
    want = [t.clone() for t in seq.backward(grad, mu, chol, amp)]

    b = FieldBatch(shapes, ids_capacity=cap)
    b.ids.fill_(-7)  # any id the backward reads must come from the BIN stage, not from a racing render
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    for _ in range(3):  # repeated steps reuse both workspaces
        b.forward_stages(mu, chol, amp, _lib.GF_STAGE_BIN, main)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            got = b.backward(grad, mu, chol, amp, stream=side)
        b.forward_stages(mu, chol, amp, _lib.GF_STAGE_RENDER, main)
        main.wait_stream(side)
        torch.cuda.synchronize()
        assert torch.equal(b.delta, want_delta)
        for g, w in zip(got, want):
            assert torch.equal(g, w)
    assert b.device_flags() == 0


def test_field_range_renders_equal_the_full_forward():
    """BIN once, then gf_forward_render_fields over disjoint ranges (the
    multi-GPU schedule) into per-field outputs scattered in a larger buffer:
    every field's delta equals the full forward's bit for bit, and the
    untouched gaps keep their fill."""
    shapes, (mu, chol, amp, grad), cap = _setup()
    a = FieldBatch(shapes, ids_capacity=cap)
    want = a.forward(mu, chol, amp).clone()
    numels = [o * i for o, i, _ in shapes]
    gap = 64
    buf = torch.full((sum(numels) + gap * len(shapes),), 7.0, dtype=torch.bfloat16, device="cuda")
    outs, off = [], 0
    for n in numels:
        off += gap
        outs.append(buf[off:off + n])
        off += n
    b = FieldBatch(shapes, ids_capacity=cap, field_outputs=outs)
    b.forward_stages(mu, chol, amp, _lib.GF_STAGE_BIN)
    for first, count in ((0, 5), (5, 1), (6, 11), (17, 7)):
        b.forward_render_fields(mu, chol, amp, first, count)
    torch.cuda.synchronize()
    for f in range(len(shapes)):
        assert torch.equal(b.delta_view(f).reshape(-1), want[a.n_off[f]:a.n_off[f + 1]]), f
    off = 0
    for n in numels:
        assert bool((buf[off:off + gap] == 7.0).all())
        off += gap + n
    got = b.backward(grad, mu, chol, amp)
    ref = a.backward(grad, mu, chol, amp)
    for g, r in zip(got, ref):
        assert torch.equal(g, r)
    assert a.device_flags() == 0 and b.device_flags() == 0


def test_field_range_arguments_are_checked():
    shapes, (mu, chol, amp, grad), cap = _setup()
    b = FieldBatch(shapes, ids_capacity=cap)
    b.forward_stages(mu, chol, amp, _lib.GF_STAGE_BIN)
    for first, count in ((-1, 2), (0, 0), (20, 5)):
        with pytest.raises(_lib.GfieldError, match="field range"):
            b.forward_render_fields(mu, chol, amp, first, count)
