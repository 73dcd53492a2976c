"""Densified layers (K in the thousands) on one B200.

GUASS's densify controller clones and splits Gaussians during training
(gaussian_peft/trainers/base_trainer.py:127-220), so a layer's K grows far
beyond its initial 256.  The binning here rebuilds each tile's list by a
candidate scan over the field's K boxes instead of the reference's global
radix sort (forward.cu:99-132, 211-241); these tests hold it to the same bar
at K = 4096 and 16384 on a 1280x1280 field: bins and ids bit-exact against the
oracle and the reference's own extension, fp32 delta bit-identical to the
reference extension's, gradients within the condition-aware bound.  The
drop-in training path reserves no K x T id buffer: its memory follows the
pair count, and a pair count that outgrows the previous call's is re-binned.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from guass_b200 import synthetic as S
from gpu_helpers import (PARITY_LOG, assert_grads_exact_within, exact_grads, reference_undefined_tiles, run_ext,
                         tile_mask_to_elements)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_ext():
    try:
        from oracle import build_ref
        return build_ref.load()
    except (FileNotFoundError, ImportError, OSError):
        return None


@pytest.mark.parametrize("k", [4096, 16384])
def test_densified_field_bit_exact(ref_ext, k):
    import oracle

    f = S.densified(k)
    delta, tp, ids, grads = run_ext(f)
    o_delta, o_tp, o_ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp)
    np.testing.assert_array_equal(tp, o_tp)
    np.testing.assert_array_equal(ids, o_ids)
    np.testing.assert_allclose(delta, o_delta, rtol=1e-5, atol=max(1e-7, 2e-6 * float(np.abs(o_delta).max())))
    assert_grads_exact_within(grads, exact_grads(f, tp, ids), label=f"dense{k}:")
    if ref_ext is None:
        return
    d = f.to("cuda")
    r_delta, r_tp, r_ids = ref_ext.gaussian_field_forward(d.row_coords, d.col_coords, d.mu, d.chol_raw, d.amp, 32,
                                                          32, 3.0, False, 80.0)
    np.testing.assert_array_equal(tp, r_tp.cpu().numpy())
    np.testing.assert_array_equal(ids, r_ids.cpu().numpy())
    undefined = tile_mask_to_elements(reference_undefined_tiles(f.out_features, f.in_features, 32, 32, tp),
                                      f.out_features, f.in_features, 32, 32)
    differ = delta.view(np.uint32) != r_delta.cpu().numpy().view(np.uint32)
    assert not (differ & ~undefined).any()


def _train_step(f, ext=None):
    from guass_b200 import cuda_field

    d = f.to("cuda")
    mu, chol, amp = (t.clone().requires_grad_(True) for t in (d.mu, d.chol_raw, d.amp))
    delta = cuda_field.gaussian_field_train(row_coords=d.row_coords, col_coords=d.col_coords, mu=mu, chol_raw=chol,
                                            amp=amp, tile_out=32, tile_in=32, sigma_multiplier=3.0)
    delta.backward(d.grad)
    torch.cuda.synchronize()
    return delta.detach(), [t.grad.detach().clone() for t in (mu, chol, amp)]


def test_training_path_memory_follows_the_pair_count():
    """gaussian_field_train at K=16384 on 1280x1280: the reference protocol
    (exact ids, host read) and the training path give the same delta and
    gradients bit for bit; the training path's peak memory stays a small
    multiple of the pair buffers (the K x T bound would be 26 M pairs, about
    1 GB of ids and partials); and a call whose pairs outgrow the previous
    call's buffer re-bins and still matches."""
    from guass_b200.cuda_field import load_extension

    f = S.densified(16384)
    ext = load_extension()
    d = f.to("cuda")
    want_delta, tp, ids = ext.gaussian_field_forward(d.row_coords, d.col_coords, d.mu, d.chol_raw, d.amp, 32, 32,
                                                     3.0, False, 80.0)
    want = ext.gaussian_field_backward(d.grad, d.row_coords, d.col_coords, d.mu, d.chol_raw, d.amp, tp, ids, 32, 32,
                                       3.0, False, 80.0)
    pairs = int(ids.numel())
    _train_step(f)  # first call: sizes the id buffer from a default, then remembers the count
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    delta, grads = _train_step(f)
    peak = torch.cuda.max_memory_allocated() - base
    assert torch.equal(delta, want_delta)
    for g, w in zip(grads, want):
        assert torch.equal(g, w)
    field_bytes = f.numel * 4 * 2  # fp32 delta + dL/d(delta)
    bound_bytes = 40 * 16384 * 1600  # ids + partials at the K x T bound
    assert peak < field_bytes + 40 * pairs * 2 + (8 << 20), (peak, pairs)
    if PARITY_LOG:
        with open(PARITY_LOG, "a") as fh:
            fh.write(json.dumps({"case": "dense16384:train_path_memory", "pairs": pairs, "peak_bytes": peak,
                                 "k_times_t_bound_bytes": bound_bytes}) + "\n")
    # a pair count above the remembered one: the forward's id buffer overflows, the backward re-bins
    key = next(k for k in ext._train_hint if k[1:4] == (1280, 1280, 16384))
    ext._train_hint[key] = 10
    delta2, grads2 = _train_step(f)
    assert torch.equal(delta2, want_delta)
    for g, w in zip(grads2, want):
        assert torch.equal(g, w)
    assert ext._train_hint[key] == pairs


@pytest.mark.parametrize("shape,tiles", [((1000, 700), (32, 32)), ((1000, 700), (16, 24)), ((333, 2100), (32, 32))])
def test_super_tile_lists_on_ragged_grids(shape, tiles):
    """K >= 2048 takes the candidates from super-tile lists: tile grids that
    are not multiples of the super-tile, and the generic-tile render, still
    give the oracle's bins and ids bit for bit."""
    import oracle

    f = S.make_field(shape[0], shape[1], 3000, seed=21, log_scale_mean=np.log(0.015), log_scale_std=0.4,
                     elongated_frac=0.25, blob_frac=0.3)
    delta, tp, ids, grads = run_ext(f, tile_out=tiles[0], tile_in=tiles[1])
    o_delta, o_tp, o_ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tile_out=tiles[0],
                                          tile_in=tiles[1])
    np.testing.assert_array_equal(tp, o_tp)
    np.testing.assert_array_equal(ids, o_ids)
    np.testing.assert_allclose(delta, o_delta, rtol=1e-5, atol=max(1e-7, 2e-6 * float(np.abs(o_delta).max())))
    assert_grads_exact_within(grads, exact_grads(f, tp, ids, tile_out=tiles[0], tile_in=tiles[1]),
                              label=f"lists{shape}{tiles}:")


def test_super_tile_lists_with_staged_forward():
    """BIN alone writes the id lists (emit_ids_kernel, from the super-tile
    lists too); RENDER after it gives the one-call forward's delta."""
    from guass_b200 import _lib
    from guass_b200.batched import FieldBatch, pack_fields

    fields = [S.densified(4096), S.cfg1()]
    shapes = [(f.out_features, f.in_features, f.k) for f in fields]
    mu, chol, amp, _ = pack_fields(fields, device="cuda")
    a = FieldBatch(shapes, out_dtype=torch.float32)
    b = FieldBatch(shapes, out_dtype=torch.float32)
    for x in (a, b):
        while x.ensure_capacity(mu, chol, amp):
            pass
    want = a.forward(mu, chol, amp).clone()
    b.ids.fill_(-5)
    b.forward_stages(mu, chol, amp, _lib.GF_STAGE_BIN)
    ids_bin = b.ids[:b.total_pairs()].clone()
    b.forward_stages(mu, chol, amp, _lib.GF_STAGE_RENDER)
    assert torch.equal(b.delta, want)
    assert torch.equal(ids_bin, a.ids[:a.total_pairs()])
    assert a.device_flags() == 0 and b.device_flags() == 0
