"""The C ABI boundary: symbols, struct layout and host-side argument checks.

These run without a GPU: loading libgfield.so and every validation path before
the first CUDA call are host-only.
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from guass_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "gfield.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*[\w\s\*]*?\b(gf_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_entry_points():
    assert set(declared_functions()) == set(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (gf_\w+)", out))
    assert set(declared_functions()) <= exported


def test_abi_version():
    assert _lib.lib().gf_abi_version() == _lib.GF_ABI_VERSION


def test_struct_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(r'''
#include <stdio.h>
#include <stddef.h>
#include "gfield.h"
#define F(T, m) printf(#T "." #m " %zu\n", offsetof(T, m));
int main(void) {
  printf("gf_config %zu\n", sizeof(gf_config));
  printf("gf_field %zu\n", sizeof(gf_field));
  printf("gf_batch %zu\n", sizeof(gf_batch));
  printf("gf_stats_layer %zu\n", sizeof(gf_stats_layer));
  F(gf_config, clamp_quad) F(gf_config, out_scale) F(gf_config, grad_dtype) F(gf_config, flags)
  F(gf_field, row_coords) F(gf_field, ids_capacity) F(gf_field, d_amp) F(gf_field, base_weight) F(gf_field, delta_multicast)
  F(gf_batch, fields) F(gf_batch, ids_capacity) F(gf_batch, pair_base)
  F(gf_stats_layer, d_mu_raw) F(gf_stats_layer, amp) F(gf_stats_layer, stats)
  return 0;
}
''')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                              check=True).stdout.split("\n") if line)
    assert int(got["gf_config"]) == ctypes.sizeof(_lib.GfConfig)
    assert int(got["gf_field"]) == ctypes.sizeof(_lib.GfField)
    assert int(got["gf_batch"]) == ctypes.sizeof(_lib.GfBatch)
    assert int(got["gf_stats_layer"]) == ctypes.sizeof(_lib.GfStatsLayer)
    for key, val in got.items():
        if "." in key:
            struct, member = key.split(".")
            cls = {"gf_config": _lib.GfConfig, "gf_field": _lib.GfField, "gf_batch": _lib.GfBatch,
                   "gf_stats_layer": _lib.GfStatsLayer}[struct]
            assert getattr(cls, member).offset == int(val), key


def _cfg(**kw):
    base = dict(tile_out=32, tile_in=32, sigma_multiplier=3.0, normalize=0, has_clamp_quad=1, clamp_quad=80.0,
                out_scale=1.0, out_dtype=_lib.GF_F32, grad_dtype=_lib.GF_F32)
    base.update(kw)
    return _lib.GfConfig(**base)


def _batch(n=1, **field_kw):
    fields = (_lib.GfField * max(n, 1))()
    for f in fields:
        f.out_features, f.in_features, f.num_gaussians = 320, 768, 256
        for k, v in field_kw.items():
            setattr(f, k, v)
    return _lib.GfBatch(num_fields=n, fields=ctypes.cast(fields, ctypes.POINTER(_lib.GfField))), fields


def test_num_tiles():
    L = _lib.lib()
    assert L.gf_num_tiles(320, 768, 32, 32) == 240
    assert L.gf_num_tiles(70, 45, 16, 8) == 5 * 6
    assert L.gf_num_tiles(0, 5, 32, 32) == 0


def test_workspace_bytes():
    L = _lib.lib()
    b, keep = _batch()
    fwd = L.gf_workspace_bytes(ctypes.byref(_cfg()), ctypes.byref(b), _lib.GF_PASS_FORWARD)
    assert fwd >= 256 + 256 * (32 + 16)
    b.fields[0].ids_capacity = 10000
    bwd = L.gf_workspace_bytes(ctypes.byref(_cfg()), ctypes.byref(b), _lib.GF_PASS_BACKWARD)
    assert bwd >= fwd + 32 * 10000
    assert L.gf_workspace_bytes(ctypes.byref(_cfg(tile_out=0)), ctypes.byref(b), _lib.GF_PASS_FORWARD) == 0


@pytest.mark.parametrize("cfg_kw,batch_n,msg", [
    (dict(tile_out=0), 1, "tile_out must be positive"),
    (dict(tile_in=-1), 1, "tile_in must be positive"),
    (dict(sigma_multiplier=0.0), 1, "sigma_multiplier must be positive"),
    (dict(out_dtype=7), 1, "out_dtype"),
    (dict(flags=0x80000000), 1, "unknown gf_config.flags"),
    ({}, 0, "num_fields"),
    ({}, _lib.GF_MAX_FIELDS + 1, "num_fields"),
])
def test_forward_rejects_bad_arguments(cfg_kw, batch_n, msg):
    L = _lib.lib()
    b, keep = _batch(batch_n)
    st = L.gf_forward(ctypes.byref(_cfg(**cfg_kw)), ctypes.byref(b), None, 0, None)
    assert st == _lib.GF_ERR_INVALID_ARG
    assert msg in _lib.last_error()


def test_forward_rejects_null_inputs_and_small_workspace():
    L = _lib.lib()
    b, keep = _batch()
    st = L.gf_forward(ctypes.byref(_cfg()), ctypes.byref(b), None, 0, None)
    assert st == _lib.GF_ERR_INVALID_ARG and "must be non-null" in _lib.last_error()
    fake = 1 << 20  # never dereferenced: the size check fails first
    b2, keep2 = _batch(row_coords=fake, col_coords=fake, mu=fake, chol_raw=fake, amp=fake, delta=fake,
                       tile_ptr=fake, gaussian_ids=fake, ids_capacity=100)
    st = L.gf_forward(ctypes.byref(_cfg()), ctypes.byref(b2), ctypes.c_void_p(1 << 30), 64, None)
    assert st == _lib.GF_ERR_INVALID_ARG and "workspace too small" in _lib.last_error()


def test_backward_rejects_missing_grad():
    L = _lib.lib()
    fake = 1 << 20
    b, keep = _batch(row_coords=fake, col_coords=fake, mu=fake, chol_raw=fake, amp=fake, tile_ptr=fake,
                     gaussian_ids=fake, ids_capacity=100)
    st = L.gf_backward(ctypes.byref(_cfg()), ctypes.byref(b), ctypes.c_void_p(1 << 30), 1 << 30, None)
    assert st == _lib.GF_ERR_INVALID_ARG and "grad_delta" in _lib.last_error()


def test_shared_ids_requires_pair_base():
    L = _lib.lib()
    b, keep = _batch()
    b.ids = 1 << 20
    st = L.gf_forward(ctypes.byref(_cfg()), ctypes.byref(b), None, 0, None)
    assert st == _lib.GF_ERR_INVALID_ARG and "pair_base" in _lib.last_error()


def test_grad_stats_argument_errors():
    """Rejected on the host, before any device work."""
    L = _lib.lib()
    layers = (_lib.GfStatsLayer * 2)()
    assert L.gf_grad_stats_accumulate(0, None, None) == _lib.GF_OK
    assert L.gf_grad_stats_accumulate(-1, layers, None) == _lib.GF_ERR_INVALID_ARG
    assert L.gf_grad_stats_accumulate(_lib.GF_MAX_FIELDS + 1, layers, None) == _lib.GF_ERR_INVALID_ARG
    assert L.gf_grad_stats_accumulate(1, None, None) == _lib.GF_ERR_INVALID_ARG
    layers[0].num_gaussians = 4  # stats missing
    assert L.gf_grad_stats_accumulate(2, layers, None) == _lib.GF_ERR_INVALID_ARG
    assert "stats must be non-null" in _lib.last_error()
    layers[0].num_gaussians = -1
    assert L.gf_grad_stats_accumulate(1, layers, None) == _lib.GF_ERR_INVALID_ARG
    layers[0].num_gaussians = 0  # nothing to do: no launch
    assert L.gf_grad_stats_accumulate(2, layers, None) == _lib.GF_OK


def test_forward_stages_and_multicast_arguments():
    L = _lib.lib()
    fake = 1 << 20  # never dereferenced: validation fails first
    kw = dict(row_coords=fake, col_coords=fake, mu=fake, chol_raw=fake, amp=fake, delta=fake, tile_ptr=fake,
              gaussian_ids=fake, ids_capacity=100)
    b, keep = _batch(**kw)
    for bad in (0, 4, 7):
        st = L.gf_forward_stages(ctypes.byref(_cfg()), ctypes.byref(b), None, 0, bad, None)
        assert st == _lib.GF_ERR_INVALID_ARG and "stages" in _lib.last_error()
    # multicast stores need 16-byte rows: bf16 needs in_features % 8 == 0, an aligned address
    b, keep = _batch(**dict(kw, in_features=70, delta_multicast=1 << 21))
    st = L.gf_forward(ctypes.byref(_cfg(out_dtype=_lib.GF_BF16)), ctypes.byref(b), None, 0, None)
    assert st == _lib.GF_ERR_UNSUPPORTED and "delta_multicast" in _lib.last_error()
    b, keep = _batch(**dict(kw, delta_multicast=(1 << 21) + 8))
    st = L.gf_forward(ctypes.byref(_cfg(out_dtype=_lib.GF_BF16)), ctypes.byref(b), None, 0, None)
    assert st == _lib.GF_ERR_UNSUPPORTED
    b, keep = _batch(**dict(kw, delta_multicast=1 << 21))
    st = L.gf_forward(ctypes.byref(_cfg(out_dtype=_lib.GF_BF16, tile_in=12)), ctypes.byref(b), None, 0, None)
    assert st == _lib.GF_ERR_UNSUPPORTED
    # an aligned request passes validation and fails on the missing workspace instead
    st = L.gf_forward(ctypes.byref(_cfg(out_dtype=_lib.GF_BF16)), ctypes.byref(b), None, 0, None)
    assert st == _lib.GF_ERR_INVALID_ARG and "workspace" in _lib.last_error()


def test_checked_build_exports_the_same_abi():
    """libgfield_check.so (-DGF_CHECK) is a drop-in replacement of the release library."""
    from guass_b200 import _build

    lib = ctypes.CDLL(str(_build.LIB_CHECK))
    for name in _lib.EXPORTED:
        assert hasattr(lib, name), name
    lib.gf_abi_version.restype = ctypes.c_int
    assert lib.gf_abi_version() == _lib.GF_ABI_VERSION
