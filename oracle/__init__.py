"""CPU oracle for the Gaussian-field renderer (TEST INFRASTRUCTURE ONLY).

This package is the checker the CUDA product path is compared against and the
"port" CPU baseline that bench.py times.  Only tests/, ``__graft_entry__.smoke``
and bench.py's CPU-baseline leg may import it; ``guass_b200`` never does.

It wraps ``gfield_oracle.c`` (a C restatement of
``gaussian_peft/cuda_field/csrc/forward.cu`` and ``backward.cu``) through
ctypes, taking and returning numpy arrays.  :func:`build` compiles it with gcc.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SRC = _HERE / "gfield_oracle.c"
_LIB_PATH = _HERE / "libgfield_oracle.so"
_lib = None

_F = ctypes.POINTER(ctypes.c_float)
_I = ctypes.POINTER(ctypes.c_int64)
_i64 = ctypes.c_int64
_d = ctypes.c_double
_int = ctypes.c_int


def build(force: bool = False) -> Path:
    """Compile the C restatement into ``oracle/libgfield_oracle.so``."""
    if _LIB_PATH.exists() and not force and _LIB_PATH.stat().st_mtime >= _SRC.stat().st_mtime:
        return _LIB_PATH
    cmd = [
        "gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp",
        "-ffp-contract=off", "-fno-fast-math",
        str(_SRC), "-o", str(_LIB_PATH), "-lm",
    ]
    subprocess.run(cmd, check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(_LIB_PATH))
    lib.gfo_preprocess.argtypes = [_i64, _i64, _i64, _i64, _i64, _d, _F, _F, _F, _F, _I, _I, _I, _I, _I]
    lib.gfo_preprocess.restype = None
    lib.gfo_count_pairs.argtypes = [_i64, _I]
    lib.gfo_count_pairs.restype = _i64
    lib.gfo_bin.argtypes = [_i64, _i64, _i64, _I, _I, _I, _I, _I, _I]
    lib.gfo_bin.restype = None
    lib.gfo_forward.argtypes = [_i64, _i64, _i64, _i64, _F, _F, _F, _F, _F, _F, _I, _I, _int, _int, _d, _F]
    lib.gfo_forward.restype = None
    lib.gfo_backward.argtypes = [_i64, _i64, _i64, _i64, _i64, _d, _F, _F, _F, _F, _F, _F, _I, _I, _i64,
                                 _int, _int, _d, _F, _F, _F]
    lib.gfo_backward.restype = None
    _D = ctypes.POINTER(ctypes.c_double)
    lib.gfo_backward_f64.argtypes = [_i64, _i64, _i64, _i64, _i64, _d, _F, _F, _F, _F, _F, _F, _I, _I, _i64,
                                     _int, _int, _d, _D, _D, _D, _D, _D, _D, _F, _F]
    lib.gfo_backward_f64.restype = None
    lib.gfo_max_threads.argtypes = []
    lib.gfo_max_threads.restype = _int
    lib.gfo_set_threads.argtypes = [_int]
    lib.gfo_set_threads.restype = None
    _lib = lib
    return lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i64a(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def _pf(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _pi(a: np.ndarray):
    return a.ctypes.data_as(_I)


def max_threads() -> int:
    return int(_load().gfo_max_threads())


def num_tiles(out_features: int, in_features: int, tile_out: int, tile_in: int) -> tuple[int, int]:
    return (out_features + tile_out - 1) // tile_out, (in_features + tile_in - 1) // tile_in


def preprocess(out_features, in_features, mu, chol_raw, tile_out=32, tile_in=32, sigma_multiplier=3.0):
    """forward.cu:134-209 -> dict(inv_cov[K,2,2], det[K], r0, r1, c0, c1, tiles_touched)."""
    lib = _load()
    mu = _f32(mu).reshape(-1, 2)
    chol_raw = _f32(chol_raw).reshape(-1, 3)
    k = mu.shape[0]
    inv = np.zeros((k, 4), np.float32)
    det = np.zeros(k, np.float32)
    box = np.zeros((5, k), np.int64)
    lib.gfo_preprocess(out_features, in_features, k, tile_out, tile_in, float(sigma_multiplier),
                       _pf(mu), _pf(chol_raw), _pf(inv), _pf(det),
                       _pi(box[0]), _pi(box[1]), _pi(box[2]), _pi(box[3]), _pi(box[4]))
    return {"inv_cov": inv.reshape(k, 2, 2), "det": det, "r0": box[0], "r1": box[1],
            "c0": box[2], "c1": box[3], "tiles_touched": box[4]}


def bin_pairs(out_features, in_features, geom, tile_out=32, tile_in=32):
    """Stable binning (forward.cu:211-252,428-511) -> (tile_ptr[T+1], ids[P])."""
    lib = _load()
    ntr, ntc = num_tiles(out_features, in_features, tile_out, tile_in)
    k = geom["r0"].shape[0]
    p = int(lib.gfo_count_pairs(k, _pi(geom["tiles_touched"])))
    tile_ptr = np.zeros(ntr * ntc + 1, np.int64)
    ids = np.zeros(max(p, 1), np.int64)
    lib.gfo_bin(k, ntr, ntc, _pi(geom["r0"]), _pi(geom["r1"]), _pi(geom["c0"]), _pi(geom["c1"]),
                _pi(tile_ptr), _pi(ids))
    return tile_ptr, ids[:p].copy()


def forward(row_coords, col_coords, mu, chol_raw, amp, tile_out=32, tile_in=32, sigma_multiplier=3.0,
            normalize=False, clamp_quad=80.0):
    """Reference protocol forward: (delta[out*in] f32, tile_ptr i64, gaussian_ids_sorted i64)."""
    lib = _load()
    row = _f32(row_coords)
    col = _f32(col_coords)
    mu = _f32(mu).reshape(-1, 2)
    chol_raw = _f32(chol_raw).reshape(-1, 3)
    amp = _f32(amp).reshape(-1)
    out_f, in_f = row.shape[0], col.shape[0]
    geom = preprocess(out_f, in_f, mu, chol_raw, tile_out, tile_in, sigma_multiplier)
    tile_ptr, ids = bin_pairs(out_f, in_f, geom, tile_out, tile_in)
    inv = np.ascontiguousarray(geom["inv_cov"].reshape(-1))
    delta = np.zeros(out_f * in_f, np.float32)
    ids_buf = ids if ids.size else np.zeros(1, np.int64)
    lib.gfo_forward(out_f, in_f, tile_out, tile_in, _pf(row), _pf(col), _pf(mu), _pf(amp), _pf(inv),
                    _pf(geom["det"]), _pi(tile_ptr), _pi(ids_buf), int(bool(normalize)),
                    int(clamp_quad is not None), float(clamp_quad or 0.0), _pf(delta))
    return delta, tile_ptr, ids


def backward(grad_delta, row_coords, col_coords, mu, chol_raw, amp, tile_ptr, gaussian_ids_sorted,
             tile_out=32, tile_in=32, sigma_multiplier=3.0, normalize=False, clamp_quad=80.0):
    """Reference protocol backward -> (d_mu[K,2], d_chol_raw[K,3], d_amp[K,1])."""
    lib = _load()
    grad = _f32(grad_delta).reshape(-1)
    row = _f32(row_coords)
    col = _f32(col_coords)
    mu = _f32(mu).reshape(-1, 2)
    chol_raw = _f32(chol_raw).reshape(-1, 3)
    amp = _f32(amp).reshape(-1)
    tile_ptr = _i64a(tile_ptr)
    ids = _i64a(gaussian_ids_sorted)
    k = mu.shape[0]
    d_mu = np.zeros((k, 2), np.float32)
    d_chol = np.zeros((k, 3), np.float32)
    d_amp = np.zeros(k, np.float32)
    ids_buf = ids if ids.size else np.zeros(1, np.int64)
    lib.gfo_backward(row.shape[0], col.shape[0], k, tile_out, tile_in, float(sigma_multiplier), _pf(grad),
                     _pf(row), _pf(col), _pf(mu), _pf(chol_raw), _pf(amp), _pi(tile_ptr), _pi(ids_buf),
                     ids.size, int(bool(normalize)), int(clamp_quad is not None), float(clamp_quad or 0.0),
                     _pf(d_mu), _pf(d_chol), _pf(d_amp))
    return d_mu, d_chol, d_amp.reshape(k, 1)


def backward_f64(grad_delta, row_coords, col_coords, mu, chol_raw, amp, tile_ptr, gaussian_ids_sorted,
                 tile_out=32, tile_in=32, sigma_multiplier=3.0, normalize=False, clamp_quad=80.0, geometry=None):
    """Checker backward: exact (double) reductions and chain on the reference's
    float per-element terms.  Returns ((d_mu, d_chol_raw, d_amp), (S_mu, S_chol_raw, S_amp))
    where S is the same computation on absolute values (the conditioning scale).

    ``geometry`` = (inv_cov [K,2,2] float32, det [K] float32) evaluates the
    terms with a device's own preprocess instead of the host's (the host's
    log1pf/expf may differ from CUDA's by an ulp; the det cancellation of an
    elongated Gaussian turns that into ~1e-5 of its inverse covariance)."""
    lib = _load()
    grad = _f32(grad_delta).reshape(-1)
    row = _f32(row_coords)
    col = _f32(col_coords)
    mu = _f32(mu).reshape(-1, 2)
    chol_raw = _f32(chol_raw).reshape(-1, 3)
    amp = _f32(amp).reshape(-1)
    tile_ptr = _i64a(tile_ptr)
    ids = _i64a(gaussian_ids_sorted)
    k = mu.shape[0]
    outs = [np.zeros((k, 2)), np.zeros((k, 3)), np.zeros(k), np.zeros((k, 2)), np.zeros((k, 3)), np.zeros(k)]
    ids_buf = ids if ids.size else np.zeros(1, np.int64)
    P = ctypes.POINTER(ctypes.c_double)
    g_inv = g_det = None
    if geometry is not None:
        g_inv = _f32(geometry[0]).reshape(-1)
        g_det = _f32(geometry[1]).reshape(-1)
        if g_inv.size != 4 * k or g_det.size != k:
            raise ValueError("geometry must be (inv_cov [K,2,2], det [K])")
    lib.gfo_backward_f64(row.shape[0], col.shape[0], k, tile_out, tile_in, float(sigma_multiplier), _pf(grad),
                         _pf(row), _pf(col), _pf(mu), _pf(chol_raw), _pf(amp), _pi(tile_ptr), _pi(ids_buf),
                         ids.size, int(bool(normalize)), int(clamp_quad is not None), float(clamp_quad or 0.0),
                         *[o.ctypes.data_as(P) for o in outs],
                         _pf(g_inv) if g_inv is not None else None, _pf(g_det) if g_det is not None else None)
    return (outs[0], outs[1], outs[2].reshape(k, 1)), (outs[3], outs[4], outs[5].reshape(k, 1))


def set_threads(n: int) -> None:
    """Set the OpenMP thread count of subsequent calls (any time, through the
    library; the environment variable alone is read only once, at start-up)."""
    os.environ["OMP_NUM_THREADS"] = str(int(n))
    _load().gfo_set_threads(int(n))
