"""Batched all-layer renderer: every patched projection in one set of launches.

The reference renders each ``GaussianLinear`` separately
(gaussian_peft/layers/gaussian_linear.py:178-190), paying about 15 launches and
one host sync per layer in the forward and about 40 launches and 6 syncs in the
backward.  :class:`FieldBatch` renders a fixed set of fields (for example the
128 attention projections of an SD1.5 UNet) with 2 forward and 3 backward
launches in total and no host synchronisation.

Packed layout (all on one device):
  parameters  mu [sum K, 2], chol_raw [sum K, 3], amp [sum K, 1]   (field f at rows g_off[f]:)
  outputs     delta [sum out*in] (bf16 by default)                  (field f at n_off[f]:)
  binning     tile_ptr [sum (T+1)], ids [capacity], pair_base [n+1]
  gradients   d_mu, d_chol_raw, d_amp with the parameters' layout
  base_weight optional [sum out*in] out_dtype: delta becomes W0 + out_scale*value
The flat parameter/gradient layout is also what the data-parallel path
all-reduces as one buffer.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from guass_b200 import _lib
from guass_b200.cuda_field._ext import make_config

_DT = {torch.float32: _lib.GF_F32, torch.bfloat16: _lib.GF_BF16}


@dataclass(frozen=True)
class FieldShape:
    out_features: int
    in_features: int
    num_gaussians: int


class FieldBatch:
    """A fixed set of fields rendered together (at most GF_MAX_FIELDS)."""

    def __init__(self, shapes, *, tile_out: int = 32, tile_in: int = 32, sigma_multiplier: float = 3.0,
                 normalize: bool = False, clamp_quad: float | None = 80.0, out_dtype=torch.bfloat16,
                 grad_dtype=torch.float32, out_scale: float = 1.0, device="cuda", ids_capacity: int | None = None,
                 row_coords=None, col_coords=None, delta_out: torch.Tensor | None = None,
                 base_weight: torch.Tensor | None = None, delta_multicast: int | None = None,
                 bwd_exp2: bool = False, fwd_exp2: bool = False, field_outputs=None):
        self.shapes = [s if isinstance(s, FieldShape) else FieldShape(*s) for s in shapes]
        n = len(self.shapes)
        if not 1 <= n <= _lib.GF_MAX_FIELDS:
            raise ValueError(f"a batch holds 1..{_lib.GF_MAX_FIELDS} fields, got {n}")
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.tile_out, self.tile_in = int(tile_out), int(tile_in)
        self.out_dtype, self.grad_dtype = out_dtype, grad_dtype
        self.out_scale = float(out_scale)
        # bwd_exp2 / fwd_exp2: backward basis / bf16 forward basis from the base-2 hardware
        # approximation (GF_CFG_BWD_EXP2 / GF_CFG_FWD_EXP2); tolerance-bound, not bit-exact
        flags = (_lib.GF_CFG_BWD_EXP2 if bwd_exp2 else 0) | (_lib.GF_CFG_FWD_EXP2 if fwd_exp2 else 0)
        self.cfg = make_config(tile_out, tile_in, sigma_multiplier, normalize, clamp_quad,
                               out_dtype=_DT[out_dtype], grad_dtype=_DT[grad_dtype], out_scale=out_scale,
                               flags=flags)
        self._lib = _lib.lib()
        L = self._lib
        self.num_tiles = [int(L.gf_num_tiles(s.out_features, s.in_features, tile_out, tile_in)) for s in self.shapes]
        self.g_off, self.n_off, self.t_off, self.r_off, self.c_off = [0], [0], [0], [0], [0]
        for s, t in zip(self.shapes, self.num_tiles):
            self.g_off.append(self.g_off[-1] + s.num_gaussians)
            self.n_off.append(self.n_off[-1] + s.out_features * s.in_features)
            self.t_off.append(self.t_off[-1] + t + 1)
            self.r_off.append(self.r_off[-1] + s.out_features)
            self.c_off.append(self.c_off[-1] + s.in_features)
        dev = self.device
        # axes: linspace(-1, 1) per field (gaussian_peft/kernels/coords.py:37-50) unless given
        if row_coords is None:
            row_coords = [torch.linspace(-1.0, 1.0, s.out_features, dtype=torch.float32) for s in self.shapes]
        if col_coords is None:
            col_coords = [torch.linspace(-1.0, 1.0, s.in_features, dtype=torch.float32) for s in self.shapes]
        self.row = torch.cat([r.reshape(-1).float().cpu() for r in row_coords]).to(dev)
        self.col = torch.cat([c.reshape(-1).float().cpu() for c in col_coords]).to(dev)
        # field_outputs: one contiguous out_dtype tensor per field (out*in elements each, anywhere in
        # memory) that the forward writes instead of a packed delta; ``self.delta`` is then None
        self._field_out = None
        self._esz_out = torch.empty(0, dtype=out_dtype).element_size()
        if field_outputs is not None:
            if delta_out is not None or delta_multicast:
                raise ValueError("field_outputs excludes delta_out and delta_multicast")
            outs = list(field_outputs)
            if len(outs) != n:
                raise ValueError(f"field_outputs needs {n} tensors, got {len(outs)}")
            for t, sh in zip(outs, self.shapes):
                if t.dtype != out_dtype or not t.is_contiguous() or t.device != dev or \
                        t.numel() != sh.out_features * sh.in_features:
                    raise ValueError(f"each field output must be a contiguous {out_dtype} tensor of out*in "
                                     f"elements on {dev}")
            self._field_out = outs
            self.delta = None
        elif delta_out is not None:
            if delta_out.dtype != out_dtype or delta_out.numel() < self.n_off[-1] or not delta_out.is_contiguous():
                raise ValueError(f"delta_out must be a contiguous {out_dtype} tensor of >= {self.n_off[-1]} elements")
            self.delta = delta_out.view(-1)[:self.n_off[-1]]
        else:
            self.delta = torch.empty(self.n_off[-1], dtype=out_dtype, device=dev)
        self.tile_ptr = torch.empty(self.t_off[-1], dtype=torch.int64, device=dev)
        self.pair_base = torch.zeros(n + 1, dtype=torch.int64, device=dev)
        total_g = self.g_off[-1]
        cap = ids_capacity if ids_capacity is not None else 32 * total_g + 4096
        self.ids = torch.empty(max(int(cap), 1), dtype=torch.int64, device=dev)
        self.d_mu = torch.empty(total_g, 2, dtype=torch.float32, device=dev)
        self.d_chol_raw = torch.empty(total_g, 3, dtype=torch.float32, device=dev)
        self.d_amp = torch.empty(total_g, 1, dtype=torch.float32, device=dev)
        self._ws = None      # forward workspace
        self._ws_bwd = None  # backward workspace (separate, so a backward may overlap a render)
        # the last binning's pair count on its way to the host (pinned copy + event): an eager
        # backward sizes its pair partials (32 bytes per pair) by it instead of the id capacity
        self._count_host = torch.empty(1, dtype=torch.int64, pin_memory=dev.type == "cuda")
        self._count_done = None
        self._bound = None
        self._grad_bound = None
        self._out_bound = None
        self._fields = (_lib.GfField * n)()
        self._batch = _lib.GfBatch(num_fields=n, fields=ctypes.cast(self._fields, ctypes.POINTER(_lib.GfField)))
        self.base_weight = None
        if base_weight is not None:
            self.set_base_weight(base_weight)
        self.delta_multicast = None
        if delta_multicast:
            self.set_delta_multicast(delta_multicast)

    def set_delta_multicast(self, address: int | None) -> None:
        """Render through NVLink multicast: ``address`` is the multicast (NVLS)
        address of ``self.delta``'s first element; every forward then writes
        the delta of every GPU bound to that multicast object (the render and
        the all-gather in one kernel).  The caller runs a group barrier before
        any GPU reads the result.  ``None`` restores local stores."""
        self.delta_multicast = int(address) if address else None
        esz = self._esz_out
        for f in range(len(self.shapes)):
            self._fields[f].delta_multicast = None if not address else int(address) + esz * self.n_off[f]

    def set_bases(self, *, fwd_exp2: bool | None = None, bwd_exp2: bool | None = None) -> None:
        """Switch the exponential of later calls: the base-2 hardware
        approximation (GF_CFG_FWD_EXP2 for a bf16 forward, GF_CFG_BWD_EXP2 for
        the backward) or the reference's expf (False).  None keeps the current."""
        flags = int(self.cfg.flags)
        for bit, on in ((_lib.GF_CFG_FWD_EXP2, fwd_exp2), (_lib.GF_CFG_BWD_EXP2, bwd_exp2)):
            if on is not None:
                flags = (flags | bit) if on else (flags & ~bit)
        self.cfg.flags = flags

    def set_base_weight(self, base_weight: torch.Tensor | None) -> None:
        """Fused weight: later forwards store ``W0 + out_scale * value`` (one
        rounding to out_dtype) with W0 = ``base_weight`` (packed like delta;
        it may be ``self.delta`` itself).  ``None`` restores the plain delta."""
        if base_weight is not None:
            if base_weight.dtype != self.out_dtype or not base_weight.is_contiguous() \
                    or base_weight.numel() != self.numel() or base_weight.device != self.device:
                raise ValueError(f"base_weight must be a contiguous {self.out_dtype} tensor of {self.numel()} "
                                 f"elements on {self.device}")
        self.base_weight = base_weight
        esz = self._esz_out
        for f in range(len(self.shapes)):
            self._fields[f].base_weight = None if base_weight is None else base_weight.data_ptr() + esz * self.n_off[f]

    # -- parameter helpers -------------------------------------------------
    def num_fields(self) -> int:
        return len(self.shapes)

    def numel(self) -> int:
        return self.n_off[-1]

    def field_slice(self, f: int) -> slice:
        return slice(self.g_off[f], self.g_off[f + 1])

    def delta_view(self, f: int) -> torch.Tensor:
        s = self.shapes[f]
        if self._field_out is not None:
            return self._field_out[f].view(s.out_features, s.in_features)
        return self.delta[self.n_off[f]:self.n_off[f + 1]].view(s.out_features, s.in_features)

    def tile_ptr_view(self, f: int) -> torch.Tensor:
        return self.tile_ptr[self.t_off[f]:self.t_off[f + 1]]

    # -- binding -------------------------------------------------------------
    def _bind_grad(self, grad):
        if grad.dtype != self.grad_dtype or not grad.is_contiguous() or grad.numel() != self.numel() \
                or grad.device != self.device:
            raise RuntimeError(f"grad must be a contiguous {self.grad_dtype} tensor of {self.numel()} elements "
                               f"on {self.device}")
        if grad.data_ptr() == self._grad_bound:
            return
        esz = grad.element_size()
        for f in range(len(self.shapes)):
            self._fields[f].grad_delta = grad.data_ptr() + esz * self.n_off[f]
        self._grad_bound = grad.data_ptr()

    def _bind(self, mu, chol_raw, amp):
        key = (mu.data_ptr(), chol_raw.data_ptr(), amp.data_ptr(), self.ids.data_ptr())
        if key == self._bound:
            return
        total_g = self.g_off[-1]
        for name, t, cols in (("mu", mu, 2), ("chol_raw", chol_raw, 3), ("amp", amp, 1)):
            if t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.device:
                raise RuntimeError(f"{name} must be a contiguous float32 tensor on {self.device}")
            if t.numel() != total_g * cols:
                raise RuntimeError(f"{name} must have shape [{total_g}, {cols}]")
        esz_out = self._esz_out
        for f, s in enumerate(self.shapes):
            g0, n0 = self.g_off[f], self.n_off[f]
            fd = self._fields[f]
            fd.out_features, fd.in_features, fd.num_gaussians = s.out_features, s.in_features, s.num_gaussians
            fd.row_coords = self.row.data_ptr() + 4 * self.r_off[f]
            fd.col_coords = self.col.data_ptr() + 4 * self.c_off[f]
            fd.mu = mu.data_ptr() + 8 * g0
            fd.chol_raw = chol_raw.data_ptr() + 12 * g0
            fd.amp = amp.data_ptr() + 4 * g0
            fd.delta = (self._field_out[f].data_ptr() if self._field_out is not None
                        else self.delta.data_ptr() + esz_out * n0)  # rebound per call by _bind_out
            fd.tile_ptr = self.tile_ptr.data_ptr() + 8 * self.t_off[f]
            fd.gaussian_ids = None
            fd.ids_capacity = 0
            fd.d_mu = self.d_mu.data_ptr() + 8 * g0
            fd.d_chol_raw = self.d_chol_raw.data_ptr() + 12 * g0
            fd.d_amp = self.d_amp.data_ptr() + 4 * g0
        self._batch.ids = self.ids.data_ptr()
        self._batch.ids_capacity = self.ids.numel()
        self._batch.pair_base = self.pair_base.data_ptr()
        need_f = self._lib.gf_workspace_bytes(ctypes.byref(self.cfg), ctypes.byref(self._batch),
                                              _lib.GF_PASS_FORWARD)
        if need_f == 0:
            raise RuntimeError("invalid batch: " + _lib.last_error())
        if self._ws is None or self._ws.numel() < need_f:
            self._ws = torch.zeros(need_f, dtype=torch.uint8, device=self.device)
        self._bound = key
        # the loop above pointed every field at self.delta (or at its own output)
        self._out_bound = self.delta.data_ptr() if self.delta is not None else -1

    # -- passes --------------------------------------------------------------
    def forward(self, mu, chol_raw, amp, stream=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Render every field into ``self.delta`` (or into ``out``, a packed
        tensor like it, e.g. a fresh one per call so that earlier results stay
        intact); no host synchronisation."""
        return self.forward_stages(mu, chol_raw, amp, _lib.GF_STAGE_BIN | _lib.GF_STAGE_RENDER, stream, out)

    def forward_render_fields(self, mu, chol_raw, amp, first: int, count: int, stream=None) -> None:
        """The RENDER stage for fields [first, first + count) only (after a BIN
        stage of this batch): disjoint ranges may render in separate calls, so
        that an exchange of one range's delta overlaps the next range."""
        self._bind(mu, chol_raw, amp)
        self._bind_out(None)
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        _lib.check(self._lib.gf_forward_render_fields(ctypes.byref(self.cfg), ctypes.byref(self._batch),
                                                      self._ws.data_ptr(), self._ws.numel(), int(first), int(count),
                                                      st))

    def forward_stages(self, mu, chol_raw, amp, stages: int, stream=None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """``forward`` in stages (GF_STAGE_BIN, GF_STAGE_RENDER): a backward
        that needs only this step's binning may start on another stream once
        the BIN stage is done and overlap the RENDER stage."""
        self._bind(mu, chol_raw, amp)
        dst = self._bind_out(out)
        strm = stream or torch.cuda.current_stream(self.device)
        _lib.check(self._lib.gf_forward_stages(ctypes.byref(self.cfg), ctypes.byref(self._batch), self._ws.data_ptr(),
                                               self._ws.numel(), int(stages), strm.cuda_stream))
        if stages & _lib.GF_STAGE_BIN:
            self._probe_pairs(strm)
        return dst

    def _probe_pairs(self, stream):
        """Start the copy of this binning's pair count to the host (not
        inside a CUDA-graph capture, whose replays could not adapt to it)."""
        if torch.cuda.is_current_stream_capturing():
            self._count_done = None
            return
        with torch.cuda.stream(stream):
            self._count_host.copy_(self.pair_base[-1:], non_blocking=True)
            self._count_done = torch.cuda.Event()
            self._count_done.record(stream)

    def reserve_backward_workspace(self) -> None:
        """Size the backward workspace for the full id capacity now (call it
        before capturing a backward into a CUDA graph, so that the capture
        allocates and clears nothing)."""
        done, self._count_done = self._count_done, None
        self._backward_workspace()
        self._count_done = done

    # The backward's pair partials take 32 bytes per pair of capacity.  Up to
    # this size the workspace covers the whole id capacity and the backward is
    # enqueued without waiting for the forward; beyond it, eager calls size it
    # from the binning's pair count, which means waiting for that copy.
    EAGER_WORKSPACE_BUDGET = 1 << 30

    def _backward_workspace(self) -> int:
        """Size the backward workspace; returns the pair capacity to pass.
        For the whole id capacity when that fits EAGER_WORKSPACE_BUDGET (and
        under capture, where a replay may see any count); otherwise, eagerly,
        the last binning's pair count."""
        cap = self.ids.numel()
        self._batch.ids_capacity = cap
        need_b = self._lib.gf_workspace_bytes(ctypes.byref(self.cfg), ctypes.byref(self._batch),
                                              _lib.GF_PASS_BACKWARD)
        if (need_b > self.EAGER_WORKSPACE_BUDGET and self._count_done is not None
                and not torch.cuda.is_current_stream_capturing()):
            self._count_done.synchronize()
            cap = max(1, min(cap, int(self._count_host[0])))
            self._batch.ids_capacity = cap
            need_b = self._lib.gf_workspace_bytes(ctypes.byref(self.cfg), ctypes.byref(self._batch),
                                                  _lib.GF_PASS_BACKWARD)
        self._batch.ids_capacity = self.ids.numel()
        if need_b == 0:
            raise RuntimeError("invalid batch: " + _lib.last_error())
        if self._ws_bwd is None or self._ws_bwd.numel() < need_b:
            self._ws_bwd = torch.zeros(need_b, dtype=torch.uint8, device=self.device)
        return cap

    def _bind_out(self, out):
        if self._field_out is not None:
            if out is not None:
                raise RuntimeError("out= cannot be combined with field_outputs")
            return None
        dst = self.delta if out is None else out
        if out is not None and (out.dtype != self.out_dtype or not out.is_contiguous() or out.numel() != self.numel()
                                or out.device != self.device):
            raise RuntimeError(f"out must be a contiguous {self.out_dtype} tensor of {self.numel()} elements on "
                               f"{self.device}")
        if self.delta_multicast and out is not None:
            raise RuntimeError("out= cannot be combined with delta_multicast (the multicast buffer is fixed)")
        if dst.data_ptr() != self._out_bound:
            esz = dst.element_size()
            for f in range(len(self.shapes)):
                self._fields[f].delta = dst.data_ptr() + esz * self.n_off[f]
            self._out_bound = dst.data_ptr()
        return dst

    def backward(self, grad, mu, chol_raw, amp, stream=None):
        """dL/d(delta) (packed, grad_dtype) -> (d_mu, d_chol_raw, d_amp) packed."""
        self._bind(mu, chol_raw, amp)
        self._bind_grad(grad)
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        cap = self._backward_workspace()
        self._batch.ids_capacity = cap  # the backward reads ids[0, pairs) only
        try:
            _lib.check(self._lib.gf_backward(ctypes.byref(self.cfg), ctypes.byref(self._batch),
                                             self._ws_bwd.data_ptr(), self._ws_bwd.numel(), st))
        finally:
            self._batch.ids_capacity = self.ids.numel()
        return self.d_mu, self.d_chol_raw, self.d_amp

    def device_flags(self, reset: bool = True) -> int:
        """Synchronise and return the GF_FLAG_* bits recorded since the last reset."""
        out = 0
        for ws in (self._ws, self._ws_bwd):  # forward flags (capacity) and backward flags (saved state)
            if ws is None:
                continue
            flags = ctypes.c_uint32(0)
            _lib.check(self._lib.gf_workspace_status(ws.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream,
                                                     int(reset), ctypes.byref(flags)))
            out |= flags.value
        return out

    def total_pairs(self) -> int:
        return int(self.pair_base[-1].item())

    def ensure_capacity(self, mu, chol_raw, amp) -> bool:
        """Run one forward, grow the id buffer if the pairs did not fit.
        Returns True if it had to grow (the caller should render again)."""
        self.forward(mu, chol_raw, amp)
        flags = self.device_flags(reset=True)
        p = self.total_pairs()
        if p > self.ids.numel() or flags & _lib.GF_FLAG_CAPACITY:
            self.ids = torch.empty(p + p // 8 + 1024, dtype=torch.int64, device=self.device)
            self._bound = None
            return True
        return False


def pack_fields(fields, device="cuda"):
    """List of synthetic.FieldInputs -> packed (mu, chol_raw, amp, grad f32, row list, col list)."""
    mu = torch.cat([f.mu for f in fields]).to(device).contiguous()
    chol = torch.cat([f.chol_raw for f in fields]).to(device).contiguous()
    amp = torch.cat([f.amp for f in fields]).to(device).contiguous()
    grad = torch.cat([f.grad for f in fields]).to(device).contiguous()
    return mu, chol, amp, grad
