"""ctypes binding of libgfield.so (include/gfield.h).

This module loads the in-tree CUDA library and describes its C structs.  It
raises ImportError when the library is missing: there is no CPU or PyTorch
fallback for the renderer.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent
import os as _os

# GUASS_B200_LIB points at another build of the same library (development
# builds with different tuning); the default is the in-tree libgfield.so.
LIB_PATH = Path(_os.environ["GUASS_B200_LIB"]) if _os.environ.get("GUASS_B200_LIB") else PKG / "libgfield.so"

GF_ABI_VERSION = 2
GF_MAX_FIELDS = 192
GF_NOALLOC_SCRATCH_BYTES = 4 << 20

GF_OK = 0
GF_ERR_INVALID_ARG = 1
GF_ERR_CAPACITY = 2
GF_ERR_CUDA = 3
GF_ERR_STATE = 4
GF_ERR_UNSUPPORTED = 5
STATUS_NAMES = {0: "GF_OK", 1: "GF_ERR_INVALID_ARG", 2: "GF_ERR_CAPACITY", 3: "GF_ERR_CUDA",
                4: "GF_ERR_STATE", 5: "GF_ERR_UNSUPPORTED"}

GF_F32 = 0
GF_BF16 = 1
GF_PASS_FORWARD = 0
GF_PASS_BACKWARD = 1

GF_CFG_BWD_EXP2 = 0x1
GF_CFG_FWD_EXP2 = 0x2
GF_STAGE_BIN = 1
GF_STAGE_RENDER = 2
GF_FLAG_CAPACITY = 0x1
GF_FLAG_STATE = 0x2
GF_FLAG_INTERNAL = 0x4
GF_FLAG_BOUNDS = 0x8

# Every symbol include/gfield.h declares.
EXPORTED = ("gf_abi_version", "gf_last_error", "gf_num_tiles", "gf_workspace_bytes", "gf_forward",
            "gf_backward", "gf_workspace_status", "gf_trace_events", "gf_trace_count",
            "gf_forward_noalloc", "gf_multicast_store", "gf_grad_stats_accumulate",
            "gf_forward_stages", "gf_forward_render_fields")


class GfConfig(ctypes.Structure):
    _fields_ = [
        ("tile_out", ctypes.c_int64),
        ("tile_in", ctypes.c_int64),
        ("sigma_multiplier", ctypes.c_double),
        ("normalize", ctypes.c_int32),
        ("has_clamp_quad", ctypes.c_int32),
        ("clamp_quad", ctypes.c_double),
        ("out_scale", ctypes.c_float),
        ("out_dtype", ctypes.c_int32),
        ("grad_dtype", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
    ]


class GfField(ctypes.Structure):
    _fields_ = [
        ("out_features", ctypes.c_int64),
        ("in_features", ctypes.c_int64),
        ("num_gaussians", ctypes.c_int64),
        ("row_coords", ctypes.c_void_p),
        ("col_coords", ctypes.c_void_p),
        ("mu", ctypes.c_void_p),
        ("chol_raw", ctypes.c_void_p),
        ("amp", ctypes.c_void_p),
        ("delta", ctypes.c_void_p),
        ("tile_ptr", ctypes.c_void_p),
        ("gaussian_ids", ctypes.c_void_p),
        ("ids_capacity", ctypes.c_int64),
        ("grad_delta", ctypes.c_void_p),
        ("d_mu", ctypes.c_void_p),
        ("d_chol_raw", ctypes.c_void_p),
        ("d_amp", ctypes.c_void_p),
        ("base_weight", ctypes.c_void_p),
        ("delta_multicast", ctypes.c_void_p),
    ]


class GfBatch(ctypes.Structure):
    _fields_ = [
        ("num_fields", ctypes.c_int32),
        ("fields", ctypes.POINTER(GfField)),
        ("ids", ctypes.c_void_p),
        ("ids_capacity", ctypes.c_int64),
        ("pair_base", ctypes.c_void_p),
    ]


_lib = None


class GfStatsLayer(ctypes.Structure):
    _fields_ = [
        ("num_gaussians", ctypes.c_int64),
        ("d_mu_raw", ctypes.c_void_p),
        ("d_chol_raw", ctypes.c_void_p),
        ("d_amp", ctypes.c_void_p),
        ("amp", ctypes.c_void_p),
        ("stats", ctypes.c_void_p),
    ]


class GfieldError(RuntimeError):
    """A libgfield call returned a non-OK status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libgfield.so once; ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m guass_b200._build` "
                          "(or __graft_entry__.build()); there is no fallback implementation")
    L = ctypes.CDLL(str(LIB_PATH))
    L.gf_abi_version.restype = ctypes.c_int
    L.gf_last_error.restype = ctypes.c_char_p
    L.gf_num_tiles.argtypes = [ctypes.c_int64] * 4
    L.gf_num_tiles.restype = ctypes.c_int64
    L.gf_workspace_bytes.argtypes = [ctypes.POINTER(GfConfig), ctypes.POINTER(GfBatch), ctypes.c_int]
    L.gf_workspace_bytes.restype = ctypes.c_size_t
    for fn in (L.gf_forward, L.gf_backward):
        fn.argtypes = [ctypes.POINTER(GfConfig), ctypes.POINTER(GfBatch), ctypes.c_void_p, ctypes.c_size_t,
                       ctypes.c_void_p]
        fn.restype = ctypes.c_int
    L.gf_workspace_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_uint32)]
    L.gf_workspace_status.restype = ctypes.c_int
    L.gf_trace_events.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]
    L.gf_trace_events.restype = ctypes.c_int
    L.gf_trace_count.argtypes = []
    L.gf_trace_count.restype = ctypes.c_int
    L.gf_forward_noalloc.argtypes = [ctypes.POINTER(GfConfig), ctypes.POINTER(GfBatch), ctypes.c_void_p]
    L.gf_forward_noalloc.restype = ctypes.c_int
    L.gf_multicast_store.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    L.gf_multicast_store.restype = ctypes.c_int
    L.gf_grad_stats_accumulate.argtypes = [ctypes.c_int32, ctypes.POINTER(GfStatsLayer), ctypes.c_void_p]
    L.gf_grad_stats_accumulate.restype = ctypes.c_int
    L.gf_forward_stages.argtypes = [ctypes.POINTER(GfConfig), ctypes.POINTER(GfBatch), ctypes.c_void_p,
                                    ctypes.c_size_t, ctypes.c_uint, ctypes.c_void_p]
    L.gf_forward_stages.restype = ctypes.c_int
    L.gf_forward_render_fields.argtypes = [ctypes.POINTER(GfConfig), ctypes.POINTER(GfBatch), ctypes.c_void_p,
                                           ctypes.c_size_t, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
    L.gf_forward_render_fields.restype = ctypes.c_int
    if L.gf_abi_version() != GF_ABI_VERSION:
        raise ImportError(f"libgfield ABI {L.gf_abi_version()} != expected {GF_ABI_VERSION}")
    _lib = L
    return L


def check(status: int) -> None:
    if status != GF_OK:
        msg = lib().gf_last_error()
        raise GfieldError(status, msg.decode() if msg else "")


def last_error() -> str:
    msg = lib().gf_last_error()
    return msg.decode() if msg else ""
