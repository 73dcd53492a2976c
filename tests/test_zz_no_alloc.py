"""gf_forward_noalloc: the forward render for callers that cannot allocate.

Some callers run inside a host that owns all device memory -- an inference
engine's plugin, a framework's custom call, a runtime with a fixed memory
budget -- and are handed only their input and output buffers: they may not
call cudaMalloc and have no way to provide the scratch workspace gf_forward
takes.  gf_forward_noalloc keeps that scratch in a static array inside the
library instead.  These tests call it through the C ABI and check its outputs
against gf_forward's (with a caller workspace) on two calls in a row, so a
second call must not see leftovers of the first.

This file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from guass_b200 import _lib, synthetic
from guass_b200.cuda_field._ext import make_config

pytestmark = pytest.mark.gpu



def _batch(fields, cfg):
    """Per-field id mode batch with output buffers allocated by the test."""
    keep, descs = [], (_lib.GfField * len(fields))()
    L = _lib.lib()
    for d, f in zip(descs, fields):
        g = f.to("cuda")
        t = int(L.gf_num_tiles(f.out_features, f.in_features, cfg.tile_out, cfg.tile_in))
        cap = f.k * t
        out = dict(delta=torch.full((f.numel,), float("nan"), device="cuda"),
                   tile_ptr=torch.full((t + 1,), -7, dtype=torch.int64, device="cuda"),
                   ids=torch.full((max(cap, 1),), -7, dtype=torch.int64, device="cuda"))
        keep.append((g, out))
        d.out_features, d.in_features, d.num_gaussians = f.out_features, f.in_features, f.k
        d.row_coords, d.col_coords = g.row_coords.data_ptr(), g.col_coords.data_ptr()
        d.mu, d.chol_raw, d.amp = g.mu.data_ptr(), g.chol_raw.data_ptr(), g.amp.data_ptr()
        d.delta, d.tile_ptr = out["delta"].data_ptr(), out["tile_ptr"].data_ptr()
        d.gaussian_ids, d.ids_capacity = out["ids"].data_ptr(), cap
    b = _lib.GfBatch(num_fields=len(fields), fields=ctypes.cast(descs, ctypes.POINTER(_lib.GfField)))
    return b, descs, keep


def _outputs(keep, bf16=False):
    res = []
    for g, out in keep:
        tp = out["tile_ptr"].cpu().numpy()
        d = out["delta"]
        if bf16:  # bf16 delta fills the first half of the fp32-sized buffer
            d = d.view(torch.bfloat16)[:g.numel].float()
        res.append((d.cpu().numpy(), tp, out["ids"].cpu().numpy()[:tp[-1]]))
    return res


def _run_with_workspace(fields, cfg, bf16=False):
    L = _lib.lib()
    b, descs, keep = _batch(fields, cfg)
    n = L.gf_workspace_bytes(ctypes.byref(cfg), ctypes.byref(b), _lib.GF_PASS_FORWARD)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    _lib.check(L.gf_forward(ctypes.byref(cfg), ctypes.byref(b), ws.data_ptr(), n,
                            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return _outputs(keep, bf16)


def _run_noalloc(fields, cfg, bf16=False):
    L = _lib.lib()
    b, descs, keep = _batch(fields, cfg)
    n = L.gf_workspace_bytes(ctypes.byref(cfg), ctypes.byref(b), _lib.GF_PASS_FORWARD)
    assert n <= _lib.GF_NOALLOC_SCRATCH_BYTES
    _lib.check(L.gf_forward_noalloc(ctypes.byref(cfg), ctypes.byref(b), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return _outputs(keep, bf16)


def _assert_same(got, want):
    # both entry points launch the same kernels on the same inputs: the
    # outputs must be identical bit for bit
    for (d, tp, ids), (d0, tp0, ids0) in zip(got, want):
        np.testing.assert_array_equal(tp, tp0)
        np.testing.assert_array_equal(ids, ids0)
        assert np.isfinite(d).all()
        np.testing.assert_array_equal(d.view(np.uint32), d0.view(np.uint32))


def test_noalloc_matches_workspace_forward_two_calls_in_a_row():
    cfg = make_config(32, 32, 3.0, False, 80.0)
    first = [synthetic.cfg1(), synthetic.cfg0()]  # a two-field batch
    second = [synthetic.cfg2()]                    # then a larger single field
    want1 = _run_with_workspace(first, cfg)
    want2 = _run_with_workspace(second, cfg)
    got1 = _run_noalloc(first, cfg)
    got2 = _run_noalloc(second, cfg)
    _assert_same(got1, want1)
    _assert_same(got2, want2)


def test_noalloc_bf16_and_normalize():
    cfg = make_config(32, 32, 2.5, True, None, out_dtype=_lib.GF_BF16)
    fields = [synthetic.make_field(96, 200, 60, seed=3)]
    want = _run_with_workspace(fields, cfg, bf16=True)
    got = _run_noalloc(fields, cfg, bf16=True)
    for (d, tp, ids), (d0, tp0, ids0) in zip(got, want):
        np.testing.assert_array_equal(tp, tp0)
        np.testing.assert_array_equal(ids, ids0)
        np.testing.assert_array_equal(d.view(np.uint32), d0.view(np.uint32))


def _shared_batch(fields, cfg):
    """Shared-id mode: every field's pairs go into one id buffer at pair_base[f]."""
    L = _lib.lib()
    b, descs, keep = _batch(fields, cfg)
    cap = sum(f.k * int(L.gf_num_tiles(f.out_features, f.in_features, cfg.tile_out, cfg.tile_in)) for f in fields)
    ids = torch.full((max(cap, 1),), -7, dtype=torch.int64, device="cuda")
    pair_base = torch.full((len(fields) + 1,), -7, dtype=torch.int64, device="cuda")
    for d in descs:
        d.gaussian_ids, d.ids_capacity = None, 0
    b.ids, b.ids_capacity, b.pair_base = ids.data_ptr(), cap, pair_base.data_ptr()
    return b, descs, keep, ids, pair_base


def _run_shared(fields, cfg, noalloc):
    L = _lib.lib()
    b, descs, keep, ids, pair_base = _shared_batch(fields, cfg)
    st = torch.cuda.current_stream().cuda_stream
    if noalloc:
        _lib.check(L.gf_forward_noalloc(ctypes.byref(cfg), ctypes.byref(b), st))
    else:
        n = L.gf_workspace_bytes(ctypes.byref(cfg), ctypes.byref(b), _lib.GF_PASS_FORWARD)
        ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
        _lib.check(L.gf_forward(ctypes.byref(cfg), ctypes.byref(b), ws.data_ptr(), n, st))
    torch.cuda.synchronize()
    pb = pair_base.cpu().numpy()
    return ([(out["delta"].cpu().numpy(), out["tile_ptr"].cpu().numpy()) for _, out in keep], pb,
            ids.cpu().numpy()[:pb[-1]])


def test_noalloc_shared_ids_two_calls_in_a_row():
    """Shared-id mode uses the scratch header's completion counter (the last
    binning CTA writes pair_base); a second call must find it reset."""
    cfg = make_config(32, 32, 3.0, False, 80.0)
    fields = [synthetic.cfg1(), synthetic.make_field(64, 96, 40, seed=9), synthetic.cfg0()]
    want = _run_shared(fields, cfg, noalloc=False)
    for _ in range(2):
        got = _run_shared(fields, cfg, noalloc=True)
        np.testing.assert_array_equal(got[1], want[1])
        np.testing.assert_array_equal(got[2], want[2])
        for (d, tp), (d0, tp0) in zip(got[0], want[0]):
            np.testing.assert_array_equal(tp, tp0)
            np.testing.assert_array_equal(d.view(np.uint32), d0.view(np.uint32))


def test_noalloc_rejects_batches_beyond_the_static_scratch():
    L = _lib.lib()
    cfg = make_config(32, 32, 3.0, False, 80.0)
    fake = 1 << 20  # never dereferenced: the size check comes first
    d = (_lib.GfField * 1)()
    d[0].out_features, d[0].in_features, d[0].num_gaussians = 4096, 4096, 200_000
    for name in ("row_coords", "col_coords", "mu", "chol_raw", "amp", "delta", "tile_ptr", "gaussian_ids"):
        setattr(d[0], name, fake)
    d[0].ids_capacity = 1
    b = _lib.GfBatch(num_fields=1, fields=ctypes.cast(d, ctypes.POINTER(_lib.GfField)))
    st = L.gf_forward_noalloc(ctypes.byref(cfg), ctypes.byref(b), None)
    assert st == _lib.GF_ERR_UNSUPPORTED
    assert "static scratch" in _lib.last_error()
