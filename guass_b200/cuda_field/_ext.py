"""Torch-facing extension object with the reference pybind module's three methods.

``load_extension()`` of GUASS returns the pybind module
``gaussian_peft_cuda_field_reference`` (gaussian_peft/cuda_field/loader.py:96-109)
whose methods are defined in gaussian_peft/cuda_field/csrc/ext.cpp:9-110.  This
module provides an object with the same method names, argument order,
return protocol and error behaviour (``RuntimeError`` with the reference's
TORCH_CHECK messages), implemented on libgfield.so through its C ABI.

Differences that do not change results:
 * launches go on ``torch.cuda.current_stream()`` instead of the legacy default
   stream the reference always uses (forward.cu:58,397);
 * the backward keeps no host synchronisation; the saved-state checks the
   reference performs on the host with 4 syncs (field_impl.cu:86-108) are made
   on the device and are raised as exceptions when ``GUASS_B200_VALIDATE=1``;
 * ``grad_delta`` may also be bfloat16 (the reference requires float32).
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from guass_b200 import _lib

_VALIDATE = os.environ.get("GUASS_B200_VALIDATE", "0") not in ("", "0")


def _check_cuda(t: torch.Tensor, name: str) -> None:
    # gaussian_peft/cuda_field/csrc/common.h:8-11
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_f32(t: torch.Tensor, name: str) -> None:
    # common.h:13-16
    _check_cuda(t, name)
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32")


def _check_index(t: torch.Tensor, name: str) -> None:
    # common.h:18-24
    _check_cuda(t, name)
    if t.dtype not in (torch.int32, torch.int64):
        raise RuntimeError(f"{name} must be int32 or int64")


def _check_config(tile_out: int, tile_in: int, sigma_multiplier: float) -> None:
    # field_impl.cu:143-145
    if tile_out <= 0:
        raise RuntimeError("tile_out must be positive")
    if tile_in <= 0:
        raise RuntimeError("tile_in must be positive")
    if not sigma_multiplier > 0.0:
        raise RuntimeError("sigma_multiplier must be positive")


def _validate_forward_inputs(row_coords, col_coords, mu, chol_raw, amp) -> None:
    # field_impl.cu:52-71
    _check_f32(row_coords, "row_coords")
    _check_f32(col_coords, "col_coords")
    _check_f32(mu, "mu")
    _check_f32(chol_raw, "chol_raw")
    _check_f32(amp, "amp")
    if row_coords.dim() != 1:
        raise RuntimeError("row_coords must have shape [out_features]")
    if col_coords.dim() != 1:
        raise RuntimeError("col_coords must have shape [in_features]")
    if not (mu.dim() == 2 and mu.size(1) == 2):
        raise RuntimeError("mu must have shape [K, 2]")
    if not (chol_raw.dim() == 2 and chol_raw.size(1) == 3):
        raise RuntimeError("chol_raw must have shape [K, 3]")
    if not (amp.dim() == 2 and amp.size(1) == 1):
        raise RuntimeError("amp must have shape [K, 1]")
    if mu.size(0) != chol_raw.size(0):
        raise RuntimeError("mu and chol_raw must have the same K")
    if mu.size(0) != amp.size(0):
        raise RuntimeError("mu and amp must have the same K")
    devs = {t.device for t in (row_coords, col_coords, mu, chol_raw, amp)}
    if len(devs) != 1:
        raise RuntimeError("all inputs must be on the same CUDA device")


def make_config(tile_out, tile_in, sigma_multiplier, normalize, clamp_quad, *, out_dtype=_lib.GF_F32,
                grad_dtype=_lib.GF_F32, out_scale=1.0, flags=0) -> _lib.GfConfig:
    return _lib.GfConfig(
        tile_out=int(tile_out), tile_in=int(tile_in), sigma_multiplier=float(sigma_multiplier),
        normalize=int(bool(normalize)), has_clamp_quad=int(clamp_quad is not None),
        clamp_quad=float(clamp_quad) if clamp_quad is not None else 0.0,
        out_scale=float(out_scale), out_dtype=int(out_dtype), grad_dtype=int(grad_dtype), flags=int(flags))


class WorkspacePool:
    """One zero-initialised scratch buffer per (device, stream), grown on demand.

    Calls on one stream are ordered, so they may share its workspace."""

    def __init__(self):
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        stream = torch.cuda.current_stream(device)
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 16)
                if buf is not None:
                    size = max(size, buf.numel() * 2)
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


_POOL = WorkspacePool()


def _ptr(t) -> int | None:
    return t.data_ptr() if t is not None else None


def raise_device_flags(ws: torch.Tensor, ignore: int = 0) -> None:
    """Synchronise and raise if the device recorded an error condition
    (other than the bits in ``ignore``)."""
    flags = ctypes.c_uint32(0)
    stream = torch.cuda.current_stream(ws.device).cuda_stream
    _lib.check(_lib.lib().gf_workspace_status(ws.data_ptr(), stream, 1, ctypes.byref(flags)))
    f = flags.value & ~ignore
    if f & _lib.GF_FLAG_STATE:
        raise RuntimeError("saved tile_ptr / gaussian_ids_sorted do not match mu and chol_raw "
                           "(out-of-range, unsorted or foreign pair)")
    if f & _lib.GF_FLAG_CAPACITY:
        raise RuntimeError("gaussian id buffer too small for the pair count")
    if f & _lib.GF_FLAG_INTERNAL:
        raise RuntimeError("internal error: per-tile Gaussian list disagreed with tile_ptr")


class _PairProbe:
    """The training forward's pair count on its way to the host: a pinned
    one-element tensor, the event after its copy, the id capacity used."""

    __slots__ = ("count", "done", "capacity")

    def __init__(self, count, done, capacity):
        self.count, self.done, self.capacity = count, done, capacity


class GaussianFieldExtension:
    """Drop-in for the reference's extension module (ext.cpp:9-110)."""

    def __init__(self):
        self._lib = _lib.lib()
        self._pairs_hint: dict[tuple, int] = {}
        self._train_hint: dict[tuple, int] = {}

    # ext.cpp:9-37, field_impl.cu:135-163
    def gaussian_field_forward(self, row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in,
                               sigma_multiplier, normalize, clamp_quad):
        _validate_forward_inputs(row_coords, col_coords, mu, chol_raw, amp)
        _check_config(tile_out, tile_in, sigma_multiplier)
        return self.forward_into(row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in,
                                 sigma_multiplier, normalize, clamp_quad)

    def forward_into(self, row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in, sigma_multiplier,
                     normalize, clamp_quad, *, out_dtype=torch.float32, out_scale=1.0):
        device = mu.device
        out_f, in_f, k = row_coords.numel(), col_coords.numel(), mu.size(0)
        num_tiles = int(self._lib.gf_num_tiles(out_f, in_f, int(tile_out), int(tile_in)))
        delta = torch.empty(out_f * in_f, dtype=out_dtype, device=device)
        tile_ptr = torch.empty(num_tiles + 1, dtype=torch.int64, device=device)
        key = (out_f, in_f, k, int(tile_out), int(tile_in), float(sigma_multiplier))
        bound = k * num_tiles
        hint = self._pairs_hint.get(key, 0)
        cap = min(bound, max(hint + hint // 4 + 64, 32 * k + 1024))
        gdt = _lib.GF_BF16 if out_dtype == torch.bfloat16 else _lib.GF_F32
        cfg = make_config(tile_out, tile_in, sigma_multiplier, normalize, clamp_quad, out_dtype=gdt,
                          out_scale=out_scale)
        retried = False
        while True:
            ids = torch.empty(max(cap, 1), dtype=torch.int64, device=device)
            field = _lib.GfField(out_features=out_f, in_features=in_f, num_gaussians=k,
                                 row_coords=row_coords.data_ptr(), col_coords=col_coords.data_ptr(),
                                 mu=mu.data_ptr(), chol_raw=chol_raw.data_ptr(), amp=amp.data_ptr(),
                                 delta=delta.data_ptr(), tile_ptr=tile_ptr.data_ptr(), gaussian_ids=ids.data_ptr(),
                                 ids_capacity=cap)
            batch = _lib.GfBatch(num_fields=1, fields=ctypes.pointer(field), ids=None, ids_capacity=0,
                                 pair_base=None)
            nbytes = self._lib.gf_workspace_bytes(ctypes.byref(cfg), ctypes.byref(batch), _lib.GF_PASS_FORWARD)
            if nbytes == 0:
                _lib.check(_lib.GF_ERR_INVALID_ARG)
            with torch.cuda.device(device):
                ws = _POOL.get(device, nbytes)
                stream = torch.cuda.current_stream(device).cuda_stream
                _lib.check(self._lib.gf_forward(ctypes.byref(cfg), ctypes.byref(batch), ws.data_ptr(), ws.numel(),
                                                stream))
                # The pair count sizes the returned ids tensor: one 8-byte read
                # (the reference makes the same host round trip, forward.cu:48-73).
                num_pairs = int(tile_ptr[-1].item())
            if num_pairs <= cap:
                break
            cap = num_pairs  # rare: re-render with an exact buffer
            retried = True
        self._pairs_hint[key] = num_pairs
        if _VALIDATE:  # (a first attempt that outgrew its id buffer left the capacity bit)
            raise_device_flags(ws, ignore=_lib.GF_FLAG_CAPACITY if retried else 0)
        return delta, tile_ptr, ids[:num_pairs]

    # ext.cpp:38-72, field_impl.cu:165-179
    def gaussian_field_backward(self, grad_delta, row_coords, col_coords, mu, chol_raw, amp, tile_ptr,
                                gaussian_ids_sorted, tile_out, tile_in, sigma_multiplier, normalize, clamp_quad):
        # validate_backward_inputs (field_impl.cu:73-84); bf16 grads also accepted
        _check_cuda(grad_delta, "grad_delta")
        if grad_delta.dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError("grad_delta must be float32")
        _check_f32(row_coords, "saved.row_coords")
        _check_f32(col_coords, "saved.col_coords")
        _check_f32(mu, "saved.mu")
        _check_f32(chol_raw, "saved.chol_raw")
        _check_f32(amp, "saved.amp")
        _check_index(tile_ptr, "saved.tile_ptr")
        _check_index(gaussian_ids_sorted, "saved.gaussian_ids_sorted")
        # validate_saved_state_contract, host-side part (field_impl.cu:86-91)
        if tile_ptr.dim() != 1:
            raise RuntimeError("saved.tile_ptr must have shape [num_tiles + 1]")
        if gaussian_ids_sorted.dim() != 1:
            raise RuntimeError("saved.gaussian_ids_sorted must have shape [num_pairs]")
        if tile_ptr.numel() < 1:
            raise RuntimeError("saved.tile_ptr must contain at least one element")
        _check_config(tile_out, tile_in, sigma_multiplier)
        out_f, in_f = row_coords.numel(), col_coords.numel()
        if grad_delta.numel() != out_f * in_f:
            raise RuntimeError("grad_delta must match flattened delta shape")
        num_tiles = int(self._lib.gf_num_tiles(out_f, in_f, int(tile_out), int(tile_in)))
        if tile_ptr.numel() != num_tiles + 1:
            raise RuntimeError("saved.tile_ptr must have shape [num_tiles + 1]")
        device = mu.device
        k = mu.size(0)
        tile_ptr = tile_ptr.to(torch.int64)
        ids = gaussian_ids_sorted.to(torch.int64)
        d_mu = torch.empty(k, 2, dtype=torch.float32, device=device)
        d_chol = torch.empty(k, 3, dtype=torch.float32, device=device)
        d_amp = torch.empty(k, 1, dtype=torch.float32, device=device)
        if k == 0:
            return [d_mu, d_chol, d_amp]
        gdt = _lib.GF_BF16 if grad_delta.dtype == torch.bfloat16 else _lib.GF_F32
        cfg = make_config(tile_out, tile_in, sigma_multiplier, normalize, clamp_quad, grad_dtype=gdt)
        field = _lib.GfField(out_features=out_f, in_features=in_f, num_gaussians=k,
                             row_coords=row_coords.data_ptr(), col_coords=col_coords.data_ptr(),
                             mu=mu.data_ptr(), chol_raw=chol_raw.data_ptr(), amp=amp.data_ptr(),
                             tile_ptr=tile_ptr.data_ptr(), gaussian_ids=ids.data_ptr() if ids.numel() else None,
                             ids_capacity=ids.numel(), grad_delta=grad_delta.data_ptr(), d_mu=d_mu.data_ptr(),
                             d_chol_raw=d_chol.data_ptr(), d_amp=d_amp.data_ptr())
        batch = _lib.GfBatch(num_fields=1, fields=ctypes.pointer(field), ids=None, ids_capacity=0, pair_base=None)
        nbytes = self._lib.gf_workspace_bytes(ctypes.byref(cfg), ctypes.byref(batch), _lib.GF_PASS_BACKWARD)
        if nbytes == 0:
            _lib.check(_lib.GF_ERR_INVALID_ARG)
        with torch.cuda.device(device):
            ws = _POOL.get(device, nbytes)
            stream = torch.cuda.current_stream(device).cuda_stream
            _lib.check(self._lib.gf_backward(ctypes.byref(cfg), ctypes.byref(batch), ws.data_ptr(), ws.numel(),
                                             stream))
            if _VALIDATE:
                raise_device_flags(ws)
        return [d_mu, d_chol, d_amp]

    # Training path without host round trips in steady state.  The public
    # forward must return gaussian_ids_sorted with exactly num_pairs entries,
    # which costs one host read of the pair count per layer (the reference
    # makes the same read, forward.cu:48-73).  The autograd training function
    # only returns delta, so it keeps the binning in the library's shared-id
    # form with the pair count on the device (pair_base) and copies that count
    # to pinned host memory asynchronously.  The id buffer is sized from the
    # previous call of the same layer shape (+25 %; every Gaussian in every
    # tile is the bound, K*T ids, which for a densified layer is hundreds of
    # MB), the backward's pair partials from this call's count, read when the
    # backward runs (long after the copy completed).  If the count outgrew the
    # id buffer (first call, or a layer whose Gaussians grew), the backward
    # bins again with room before it reads the ids: the forward's delta never
    # depends on the id buffer, so it is right either way.
    _HINT_SLACK = 4096

    @staticmethod
    def _train_key(device, out_f, in_f, k, tile_out, tile_in, sigma_multiplier):
        return (device.index, out_f, in_f, k, int(tile_out), int(tile_in), float(sigma_multiplier))

    def train_forward(self, row_coords, col_coords, mu, chol_raw, amp, tile_out, tile_in, sigma_multiplier,
                      normalize, clamp_quad, capacity=None):
        _validate_forward_inputs(row_coords, col_coords, mu, chol_raw, amp)
        _check_config(tile_out, tile_in, sigma_multiplier)
        device = mu.device
        out_f, in_f, k = row_coords.numel(), col_coords.numel(), mu.size(0)
        num_tiles = int(self._lib.gf_num_tiles(out_f, in_f, int(tile_out), int(tile_in)))
        delta = torch.empty(out_f * in_f, dtype=torch.float32, device=device)
        tile_ptr = torch.empty(num_tiles + 1, dtype=torch.int64, device=device)
        pair_base = torch.zeros(2, dtype=torch.int64, device=device)
        bound = k * num_tiles
        if capacity is None:
            hint = self._train_hint.get(self._train_key(device, out_f, in_f, k, tile_out, tile_in, sigma_multiplier))
            capacity = hint + hint // 4 + self._HINT_SLACK if hint is not None else 64 * k + self._HINT_SLACK
        cap = max(1, min(bound, int(capacity)))
        ids = torch.empty(cap, dtype=torch.int64, device=device)
        cfg = make_config(tile_out, tile_in, sigma_multiplier, normalize, clamp_quad)
        field = _lib.GfField(out_features=out_f, in_features=in_f, num_gaussians=k,
                             row_coords=row_coords.data_ptr(), col_coords=col_coords.data_ptr(),
                             mu=mu.data_ptr(), chol_raw=chol_raw.data_ptr(), amp=amp.data_ptr(),
                             delta=delta.data_ptr(), tile_ptr=tile_ptr.data_ptr())
        batch = _lib.GfBatch(num_fields=1, fields=ctypes.pointer(field), ids=ids.data_ptr(), ids_capacity=cap,
                             pair_base=pair_base.data_ptr())
        nbytes = self._lib.gf_workspace_bytes(ctypes.byref(cfg), ctypes.byref(batch), _lib.GF_PASS_FORWARD)
        if nbytes == 0:
            _lib.check(_lib.GF_ERR_INVALID_ARG)
        with torch.cuda.device(device):
            ws = _POOL.get(device, nbytes)
            stream = torch.cuda.current_stream(device)
            _lib.check(self._lib.gf_forward(ctypes.byref(cfg), ctypes.byref(batch), ws.data_ptr(), ws.numel(),
                                            stream.cuda_stream))
            count = torch.empty(1, dtype=torch.int64, pin_memory=True)
            count.copy_(pair_base[1:], non_blocking=True)
            done = torch.cuda.Event()
            done.record(stream)
            if _VALIDATE:
                raise_device_flags(ws, ignore=_lib.GF_FLAG_CAPACITY)
        probe = _PairProbe(count, done, cap)
        return delta, tile_ptr, ids, pair_base, probe

    def train_backward(self, grad_delta, row_coords, col_coords, mu, chol_raw, amp, tile_ptr, ids, pair_base,
                       tile_out, tile_in, sigma_multiplier, normalize, clamp_quad, probe=None):
        _check_cuda(grad_delta, "grad_delta")
        if grad_delta.dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError("grad_delta must be float32")
        out_f, in_f, k = row_coords.numel(), col_coords.numel(), mu.size(0)
        if grad_delta.numel() != out_f * in_f:
            raise RuntimeError("grad_delta must match flattened delta shape")
        device = mu.device
        d_mu = torch.empty(k, 2, dtype=torch.float32, device=device)
        d_chol = torch.empty(k, 3, dtype=torch.float32, device=device)
        d_amp = torch.empty(k, 1, dtype=torch.float32, device=device)
        if k == 0:
            return [d_mu, d_chol, d_amp]
        n_pairs = ids.numel()
        if probe is not None:
            probe.done.synchronize()
            n_pairs = int(probe.count[0])
            self._train_hint[self._train_key(device, out_f, in_f, k, tile_out, tile_in, sigma_multiplier)] = n_pairs
            if len(self._train_hint) > 4096:
                self._train_hint.pop(next(iter(self._train_hint)))
            if n_pairs > probe.capacity:  # the forward's id buffer overflowed: bin again with room
                _, tile_ptr, ids, pair_base, _ = self.train_forward(row_coords, col_coords, mu, chol_raw, amp,
                                                                    tile_out, tile_in, sigma_multiplier, normalize,
                                                                    clamp_quad, capacity=n_pairs)
        gdt = _lib.GF_BF16 if grad_delta.dtype == torch.bfloat16 else _lib.GF_F32
        cfg = make_config(tile_out, tile_in, sigma_multiplier, normalize, clamp_quad, grad_dtype=gdt)
        field = _lib.GfField(out_features=out_f, in_features=in_f, num_gaussians=k,
                             row_coords=row_coords.data_ptr(), col_coords=col_coords.data_ptr(),
                             mu=mu.data_ptr(), chol_raw=chol_raw.data_ptr(), amp=amp.data_ptr(),
                             tile_ptr=tile_ptr.data_ptr(), grad_delta=grad_delta.data_ptr(), d_mu=d_mu.data_ptr(),
                             d_chol_raw=d_chol.data_ptr(), d_amp=d_amp.data_ptr())
        # partial slots for exactly this call's pairs (the id buffer may be larger)
        batch = _lib.GfBatch(num_fields=1, fields=ctypes.pointer(field), ids=ids.data_ptr(),
                             ids_capacity=max(1, min(n_pairs, ids.numel())), pair_base=pair_base.data_ptr())
        nbytes = self._lib.gf_workspace_bytes(ctypes.byref(cfg), ctypes.byref(batch), _lib.GF_PASS_BACKWARD)
        if nbytes == 0:
            _lib.check(_lib.GF_ERR_INVALID_ARG)
        with torch.cuda.device(device):
            ws = _POOL.get(device, nbytes)
            stream = torch.cuda.current_stream(device).cuda_stream
            _lib.check(self._lib.gf_backward(ctypes.byref(cfg), ctypes.byref(batch), ws.data_ptr(), ws.numel(),
                                             stream))
            if _VALIDATE:
                raise_device_flags(ws)
        return [d_mu, d_chol, d_amp]

    # ext.cpp:73-110.  The reference routes this to an autograd replay of the
    # forward (backward.cu:500-539) whose result is meant to equal the train
    # backward; here it is the same exact backward.
    def gaussian_field_backward_reference(self, grad_delta, row_coords, col_coords, mu, chol_raw, amp, tile_ptr,
                                          gaussian_ids_sorted, tile_out, tile_in, sigma_multiplier, normalize,
                                          clamp_quad):
        return self.gaussian_field_backward(grad_delta, row_coords, col_coords, mu, chol_raw, amp, tile_ptr,
                                            gaussian_ids_sorted, tile_out, tile_in, sigma_multiplier, normalize,
                                            clamp_quad)
