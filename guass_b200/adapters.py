"""Whole-model use of the renderer: one batched render per step, flat gradients.

The reference renders every ``GaussianLinear`` on its own, inside each layer's
forward (gaussian_peft/layers/gaussian_linear.py:162-220, 235-242).  This
module lets a model render all its adapters at once:

* :class:`BatchedFieldFunction` -- autograd over a :class:`FieldBatch`: packed
  ``(mu, chol_raw, amp)`` in, packed delta out; the backward is the batch's
  exact backward.
* :class:`BatchedAdapters` -- binds a model's Gaussian adapters (any module with
  ``mu_raw``, ``chol_raw``, ``amp``, ``in_features``, ``out_features`` and an
  ``adapter_config``, i.e. ``GaussianLinear``) to one batch.  ``render()`` packs
  the module parameters (so they stay the parameters the optimizer, the
  checkpoints and densify see), renders every delta in one launch set and
  makes each module's ``compute_delta_weight()`` return its slice.
* :func:`allreduce_adapter_grads` -- data parallelism: all adapter gradients of
  the model in ONE flat all-reduce (the reference relies on DDP's bucketed
  hooks over the same tensors, scripts/train_diffusion.py:87-91).
* :func:`adapter_state_dict` / :func:`load_adapter_state_dict` -- the
  reference's adapter checkpoint entries (gaussian_peft/checkpoints/
  state_dict.py:12-44): per module ``mu_raw``, ``chol_raw``, ``amp``,
  ``num_gaussians``, ``in_features``, ``out_features``, ``has_bias``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn


# Pair capacity: the id buffer is reserved at the exact upper bound (every
# Gaussian in every tile of its field, 8 bytes per possible pair) up to this
# many pairs (128 MB), so no pair count can overflow it; an SD1.5 UNet with
# K=256 needs 23.4 M and measures instead.  Batches above it measure their
# pair count on the first render (and on ensure_capacity()).  The backward's
# pair partials (32 bytes per pair) follow the actual pair count, not the bound.
MAX_BOUND_PAIRS = 16_000_000


def pair_bound(shapes, tile_out: int, tile_in: int) -> int:
    return sum(k * -(-o // tile_out) * -(-i // tile_in) for o, i, k in shapes)


def _capacity_kw(shapes, tile_out, tile_in):
    bound = pair_bound(shapes, tile_out, tile_in)
    return ({"ids_capacity": max(bound, 1)}, False) if bound <= MAX_BOUND_PAIRS else ({}, True)


class _PendingNorms:
    """Per-module norms on their way to the host: a non-blocking copy into
    pinned memory and an event; :meth:`get` waits for the event once."""

    def __init__(self, norms: torch.Tensor):
        if norms.is_cuda:
            self._host = torch.empty(norms.shape, dtype=norms.dtype, pin_memory=True)
            self._host.copy_(norms, non_blocking=True)
            self._event = torch.cuda.Event()
            self._event.record()
        else:
            self._host, self._event = norms, None
        self._values = None

    def get(self, f: int) -> float:
        if self._values is None:
            if self._event is not None:
                self._event.synchronize()
            self._values = self._host.tolist()
        return self._values[f]


class _LayerMetadata(dict):
    """A layer's ``last_forward_metadata`` whose ``delta_w_norm`` (a float, as
    the layer stores it) is read from :class:`_PendingNorms` on first access
    of any entry; afterwards it is a plain dict."""

    def __init__(self, base: dict, norms: _PendingNorms, f: int):
        super().__init__(base)
        self._pending = (norms, f)

    def _resolve(self):
        if self._pending is not None:
            norms, f = self._pending
            self._pending = None
            dict.__setitem__(self, "delta_w_norm", float(norms.get(f)))

    def __getitem__(self, key):
        self._resolve()
        return dict.__getitem__(self, key)

    def get(self, key, default=None):
        self._resolve()
        return dict.get(self, key, default)

    def __contains__(self, key):
        self._resolve()
        return dict.__contains__(self, key)

    def __iter__(self):
        self._resolve()
        return dict.__iter__(self)

    def __len__(self):
        self._resolve()
        return dict.__len__(self)

    def __eq__(self, other):
        self._resolve()
        return dict.__eq__(self, other)

    __hash__ = None

    def __repr__(self):
        self._resolve()
        return dict.__repr__(self)

    def keys(self):
        self._resolve()
        return dict.keys(self)

    def values(self):
        self._resolve()
        return dict.values(self)

    def items(self):
        self._resolve()
        return dict.items(self)

    def copy(self):
        self._resolve()
        return dict(dict.items(self))


class BatchedFieldFunction(torch.autograd.Function):
    """Packed render of every field of ``batch``.

    ``batch`` provides ``forward(mu, chol_raw, amp, out=...) -> delta`` and
    ``backward(grad, mu, chol_raw, amp) -> (d_mu, d_chol_raw, d_amp)``
    (:class:`guass_b200.batched.FieldBatch`).  Every render writes a fresh
    output tensor: a graph that saved an earlier render's delta (a second
    model forward before the backward, gradient accumulation) keeps its own
    values.  The caching allocator hands the freed buffer back, so in a
    one-forward-per-step loop this costs nothing."""

    @staticmethod
    def forward(ctx, batch, mu, chol_raw, amp):
        mu, chol_raw, amp = mu.contiguous(), chol_raw.contiguous(), amp.contiguous()
        delta = batch.forward(mu, chol_raw, amp, out=torch.empty_like(batch.delta))
        ctx.batch = batch
        ctx.save_for_backward(mu, chol_raw, amp)
        return delta

    @staticmethod
    def backward(ctx, grad):
        mu, chol_raw, amp = ctx.saved_tensors
        batch = ctx.batch
        want = getattr(batch, "grad_dtype", grad.dtype)
        scale = getattr(batch, "out_scale", 1.0)  # delta = out_scale * value: dL/dvalue = scale * grad
        if scale != 1.0:
            grad = grad.float() * scale
        d_mu, d_chol, d_amp = batch.backward(grad.to(want).contiguous(), mu, chol_raw, amp)
        return None, d_mu.clone(), d_chol.clone(), d_amp.clone()


class BatchedAdapters:
    """All Gaussian adapters of a model rendered by one batch per step.

    ``modules`` maps names to adapter modules (``GaussianLinear``); their
    shapes and K fix the batch: after densify changes a K,
    :meth:`shapes_changed` is true and :meth:`rebuilt` returns the binding for
    the new K.  :meth:`freeze` / :meth:`merge_into_weights` serve inference.
    ``batch_factory(shapes, **cfg)`` builds the batch (default:
    :class:`~guass_b200.batched.FieldBatch` on the modules' device).

    ``fused_weight=True`` renders ``W_eff = W0 + adapter_scale * delta``
    straight into one buffer (the renderer's fused-weight epilogue) and makes
    each module's forward a single ``F.linear(x, W_eff, bias)``, replacing the
    reference's base GEMM plus row-chunked delta GEMMs
    (gaussian_peft/layers/gaussian_linear.py:222-242).  It needs frozen base
    weights of ``out_dtype`` and one adapter_scale for all modules; call
    :meth:`refresh_base` after changing a base weight.
    """

    def __init__(self, modules: dict, batch_factory=None, out_dtype=torch.bfloat16, fused_weight: bool = False,
                 track_metadata: bool = True, fast_exp: bool = False):
        self.names = list(modules)
        self.modules = [modules[n] for n in self.names]
        if not self.modules:
            raise ValueError("no adapter modules")
        cfg = self.modules[0].adapter_config
        for m in self.modules:
            c = m.adapter_config
            if (c.tile_out, c.tile_in, c.sigma_multiplier, c.normalize_gaussian) != \
                    (cfg.tile_out, cfg.tile_in, cfg.sigma_multiplier, cfg.normalize_gaussian):
                raise ValueError("all adapters of one batch must share tile size, sigma and normalize")
        self.shapes = [(m.out_features, m.in_features, int(m.mu_raw.shape[0])) for m in self.modules]
        kw = dict(tile_out=cfg.tile_out, tile_in=cfg.tile_in, sigma_multiplier=cfg.sigma_multiplier,
                  normalize=cfg.normalize_gaussian, clamp_quad=80.0,  # gaussian_linear.py:189
                  out_dtype=out_dtype, grad_dtype=out_dtype)
        # fast_exp: both passes on the base-2 hardware exponential (GF_CFG_FWD_EXP2 for bf16
        # deltas, GF_CFG_BWD_EXP2); tolerance-bound instead of the reference's expf
        self.fast_exp = bool(fast_exp)
        if self.fast_exp:
            kw.update(fwd_exp2=True, bwd_exp2=True)
        self.fused = bool(fused_weight)
        self.track_metadata = bool(track_metadata)
        self.w0 = None
        if self.fused:
            scales = {float(m.adapter_config.adapter_scale) for m in self.modules}
            if len(scales) != 1:
                raise ValueError("fused_weight needs one adapter_scale for all modules")
            for m in self.modules:
                if m.weight.dtype != out_dtype or m.weight.requires_grad:
                    raise ValueError(f"fused_weight needs frozen base weights of {out_dtype}")
            self.w0 = torch.cat([m.weight.detach().reshape(-1) for m in self.modules]).contiguous()
            kw.update(out_scale=scales.pop(), base_weight=self.w0)
        cap_kw, self._measure = _capacity_kw(self.shapes, cfg.tile_out, cfg.tile_in)
        kw.update(cap_kw)
        if batch_factory is None:
            from guass_b200.batched import FieldBatch

            def batch_factory(shapes, **k):
                return FieldBatch(shapes, device=self.modules[0].mu_raw.device, **k)
        self._factory, self._out_dtype = batch_factory, out_dtype
        self.batch = batch_factory(self.shapes, **kw)
        self.n_off = [0]
        for o, i, _ in self.shapes:
            self.n_off.append(self.n_off[-1] + o * i)
        self._current = None
        self._orig = {}

    def _packed_params(self):
        mu = torch.cat([torch.tanh(m.mu_raw) for m in self.modules])  # gaussian_linear.py:153-154
        chol = torch.cat([m.chol_raw for m in self.modules])
        amp = torch.cat([m.amp for m in self.modules])
        return mu, chol, amp

    @torch.no_grad()
    def ensure_capacity(self) -> None:
        """Measure the current pair count and grow the id buffer to fit (one
        host synchronisation).  Needed only for batches above MAX_BOUND_PAIRS,
        whose capacity is not the exact bound: call it when the Gaussians may
        have spread (after densify, every few hundred steps)."""
        mu, chol, amp = (t.detach().contiguous() for t in self._packed_params())
        while self.batch.ensure_capacity(mu, chol, amp):
            pass
        self._measure = False

    @torch.no_grad()
    def refresh_base(self):
        """Fused mode: copy the modules' current base weights into W0."""
        if self.fused:
            self.w0.copy_(torch.cat([m.weight.detach().reshape(-1) for m in self.modules]))

    def shapes_changed(self) -> bool:
        """True when a module's K differs from the batch's (densify cloned or
        pruned Gaussians, gaussian_peft/trainers/base_trainer.py:127-220)."""
        return any(int(m.mu_raw.shape[0]) != k for m, (_, _, k) in zip(self.modules, self.shapes))

    def rebuilt(self) -> "BatchedAdapters":
        """A new binding for the modules' current K (keeps install state)."""
        fresh = BatchedAdapters(dict(zip(self.names, self.modules)), batch_factory=self._factory,
                                out_dtype=self._out_dtype, fused_weight=self.fused,
                                track_metadata=self.track_metadata, fast_exp=self.fast_exp)
        if self._orig:
            self.uninstall()
            fresh.install()
        return fresh

    @torch.no_grad()
    def freeze(self):
        """Inference: render once and serve the cached deltas until
        :meth:`unfreeze` (the reference re-renders every layer at every
        denoising step, scripts/sample_eval_10751.py:202-259)."""
        self._frozen = False
        self._frozen = [d.clone() for d in self.render()]
        self._current = self._frozen
        return self._frozen

    def unfreeze(self):
        self._frozen = None
        self._current = None

    @torch.no_grad()
    def merge_into_weights(self):
        """Inference: add each rendered delta into its module's base weight
        once (in the weight's dtype) and make ``compute_delta_weight()``
        return zeros, so the merged weight alone carries the adapter (for
        export, or for a plain ``nn.Linear`` replacement).  Undo with
        :meth:`unmerge_weights`."""
        if self.fused:
            raise RuntimeError("merge_into_weights: the fused mode already applies W0 + delta")
        deltas = self.render()
        self._merged = []
        for m, d in zip(self.modules, deltas):
            dw = d.to(m.weight.dtype)
            m.weight.add_(dw)
            self._merged.append(dw)
        self._current = [torch.zeros_like(d) for d in deltas]
        self.install()

    @torch.no_grad()
    def unmerge_weights(self):
        for m, dw in zip(self.modules, getattr(self, "_merged", [])):
            m.weight.sub_(dw)
        self._merged = []
        self._current = None

    def render(self):
        """Render every adapter's delta (autograd-connected) and return the
        list of ``[out, in]`` deltas, already multiplied by adapter_scale
        (fused mode: the effective weights W0 + adapter_scale * delta)."""
        if getattr(self, "_frozen", None):
            return self._frozen
        if self._measure:
            self.ensure_capacity()
        mu, chol, amp = self._packed_params()
        packed = BatchedFieldFunction.apply(self.batch, mu, chol, amp)
        if self.track_metadata:
            self._publish_metadata(packed.detach())
        # one split, not a slice per module: the backward of split_with_sizes is
        # a single concatenation of the modules' gradients, while every slice's
        # backward materialises a zero-filled gradient of the whole packed delta
        sizes = [self.n_off[f + 1] - self.n_off[f] for f in range(len(self.modules))]
        out = []
        for part, m in zip(torch.split(packed, sizes), self.modules):
            d = part.view(m.out_features, m.in_features)
            scale = m.adapter_config.adapter_scale
            out.append(d * scale if scale != 1.0 and not self.fused else d)
        self._current = out
        return out

    def _publish_metadata(self, packed):
        """Each module's ``last_forward_metadata`` with the keys GaussianLinear
        writes (gaussian_linear.py:196-219) and GUASS's diagnostics read
        (utils/logging.py:17-62): execution_mode, accumulate_backend and
        delta_w_norm (of the unscaled delta, as the layer computes it).  The
        norms of all layers come from one fused launch and one asynchronous
        copy to pinned host memory; the render does not wait for them: the
        first read of a module's metadata waits for that copy (the layer
        itself synchronises once per layer per forward).  The fused mode
        renders W0 + delta and reports no norm."""
        meta = {"execution_mode": "cuda_field_train", "accumulate_backend": "gfield_batched"}
        norms = None
        if not self.fused:
            views = torch.split(packed, [self.n_off[f + 1] - self.n_off[f] for f in range(len(self.modules))])
            try:
                parts = torch._foreach_norm(views, 2, dtype=torch.float32)  # one fused launch
            except (RuntimeError, TypeError):
                parts = [torch.linalg.vector_norm(v, dtype=torch.float32) for v in views]
            norms = _PendingNorms(torch.stack(list(parts)))
        for f, m in enumerate(self.modules):
            m.last_forward_metadata = _LayerMetadata(meta, norms, f) if norms is not None else dict(meta)

    def _slot(self, f):
        if self._current is None:
            raise RuntimeError("BatchedAdapters.render() must run before the model's forward")
        return self._current[f]

    def install(self):
        """Make each module's ``compute_delta_weight()`` return its slice of
        the last :meth:`render` (call ``render()`` once per step before the
        model's forward).  Fused mode: the module's forward becomes one
        ``F.linear`` with its effective weight, and ``compute_delta_weight()``
        returns ``W_eff - W0`` (for logging; off the hot path)."""
        for f, m in enumerate(self.modules):
            if id(m) in self._orig:
                continue
            self._orig[id(m)] = (m.compute_delta_weight, m.__dict__.get("forward"))
            if self.fused:
                n0, n1 = self.n_off[f], self.n_off[f + 1]

                def cdw(f=f, m=m, n0=n0, n1=n1):
                    w0 = self.w0[n0:n1].view(m.out_features, m.in_features)
                    return self._slot(f).float() - w0.float()

                def fwd(x, f=f, m=m):
                    return F.linear(x, self._slot(f), m.bias)

                m.forward = fwd
            else:
                def cdw(f=f):
                    return self._slot(f)

            m.compute_delta_weight = cdw

    def uninstall(self):
        for m in self.modules:
            orig = self._orig.pop(id(m), None)
            if orig is not None:
                m.compute_delta_weight = orig[0]
                if orig[1] is None:
                    m.__dict__.pop("forward", None)
                else:
                    m.forward = orig[1]


def gaussian_adapter_modules(model: nn.Module) -> dict:
    """``{name: module}`` of every Gaussian adapter layer of ``model`` (modules
    with ``mu_raw``, ``chol_raw``, ``amp`` and ``adapter_config``, i.e.
    GUASS's GaussianLinear)."""
    return {n: m for n, m in model.named_modules()
            if all(hasattr(m, a) for a in ("mu_raw", "chol_raw", "amp", "adapter_config"))}


class ModelRenderer:
    """Every Gaussian adapter of ``model`` served by one batched render per
    model forward (a forward pre-hook on ``model``), instead of one render per
    layer inside each layer's forward (gaussian_linear.py:162-242).

    After densify changes a layer's K the next forward rebuilds the binding.
    ``remove()`` restores the layers' own rendering.  Keyword arguments go to
    :class:`BatchedAdapters` (``out_dtype``, ``fused_weight``, ...)."""

    def __init__(self, model: nn.Module, **kw):
        mods = gaussian_adapter_modules(model)
        if not mods:
            raise ValueError("the model has no Gaussian adapter layers")
        self.bank = BatchedAdapters(mods, **kw)
        self.bank.install()
        self._handle = model.register_forward_pre_hook(self._before_forward)

    def _before_forward(self, module, args):
        if self.bank.shapes_changed():
            self.bank = self.bank.rebuilt()
        self.bank.render()

    def remove(self) -> None:
        self._handle.remove()
        self.bank.uninstall()


def adapter_parameters(modules) -> list[torch.Tensor]:
    return [p for m in modules for p in (m.mu_raw, m.chol_raw, m.amp)]


def allreduce_adapter_grads(modules, group=None, average: bool = True) -> None:
    """Sum (and average) every adapter gradient across the group with one
    flat all-reduce of the concatenated gradients."""
    params = [p for p in adapter_parameters(modules) if p.grad is not None]
    if not params:
        return
    flat = torch.cat([p.grad.reshape(-1) for p in params])
    dist.all_reduce(flat, group=group)
    if average:
        flat /= dist.get_world_size(group)
    off = 0
    for p in params:
        n = p.grad.numel()
        p.grad.copy_(flat[off:off + n].view_as(p.grad))
        off += n


def adapter_state_dict(named_modules) -> dict:
    """Reference adapter checkpoint entries for ``{name: module}``
    (gaussian_peft/checkpoints/state_dict.py:12-26)."""
    state = {}
    for name, m in named_modules.items():
        state[name] = {
            "mu_raw": m.mu_raw.detach().cpu(),
            "chol_raw": m.chol_raw.detach().cpu(),
            "amp": m.amp.detach().cpu(),
            "num_gaussians": int(m.mu_raw.shape[0]),
            "in_features": m.in_features,
            "out_features": m.out_features,
            "has_bias": getattr(m, "bias", None) is not None,
        }
    return state


def load_adapter_state_dict(named_modules, state: dict) -> None:
    """Load reference adapter entries into ``{name: module}`` (schema-checked
    like gaussian_peft/checkpoints/state_dict.py:29-84); K may differ from the
    module's current K (densify), the parameters are replaced."""
    for name, entry in state.items():
        if name not in named_modules:
            raise KeyError(f"Gaussian adapter target module {name!r} not found in model")
        m = named_modules[name]
        expected = {"in_features": m.in_features, "out_features": m.out_features,
                    "has_bias": getattr(m, "bias", None) is not None}
        actual = {k: entry[k] for k in expected}
        if expected != actual:
            raise ValueError(f"Adapter schema mismatch for {name!r}: expected {expected}, got {actual}")
        dev, dt = m.mu_raw.device, m.mu_raw.dtype
        m.mu_raw = nn.Parameter(entry["mu_raw"].to(dev, dt))
        m.chol_raw = nn.Parameter(entry["chol_raw"].to(dev, dt))
        m.amp = nn.Parameter(entry["amp"].to(dev, dt))


class CheckpointFields:
    """A saved adapter checkpoint rendered without its model.

    Takes the payload of the reference's ``save_adapter_checkpoint``
    (gaussian_peft/checkpoints/io.py:18-32: ``{"format", "step", "metadata",
    "adapters"}``) or just its ``adapters`` mapping, checks every entry like
    ``load_gaussian_adapter_state_dict`` (checkpoints/state_dict.py:29-84,
    shapes against ``num_gaussians``), and packs all modules into one batch:
    ``mu = tanh(mu_raw)`` (gaussian_linear.py:153-154), ``chol_raw``, ``amp``.
    Render settings come from ``metadata["adapter_config"]`` (tile_out,
    tile_in, sigma_multiplier, normalize_gaussian, adapter_scale), else the
    GaussianAdapterConfig defaults; keyword arguments override both.
    ``render()`` returns ``{module name: [out, in] delta * adapter_scale}``,
    or with ``base_weights`` the fused ``W0 + adapter_scale * delta``.
    """

    _DEFAULTS = dict(tile_out=32, tile_in=32, sigma_multiplier=3.0, normalize_gaussian=False, adapter_scale=1.0)

    def __init__(self, checkpoint, device="cuda", out_dtype=torch.bfloat16, batch_factory=None,
                 base_weights: dict | None = None, **overrides):
        adapters = checkpoint.get("adapters", checkpoint) if isinstance(checkpoint, dict) else None
        if not isinstance(adapters, dict) or not adapters:
            raise ValueError("no adapter entries in the checkpoint")
        meta = (checkpoint.get("metadata") or {}) if "adapters" in checkpoint else {}
        cfg = dict(self._DEFAULTS)
        cfg.update({k: v for k, v in (meta.get("adapter_config") or {}).items() if k in cfg})
        unknown = set(overrides) - set(cfg)
        if unknown:
            raise TypeError(f"unknown render settings {sorted(unknown)}")
        cfg.update(overrides)
        self.config = cfg
        self.names = list(adapters)
        self.shapes, mus, chols, amps = [], [], [], []
        for name in self.names:
            e = adapters[name]
            for key in ("mu_raw", "chol_raw", "amp", "num_gaussians", "in_features", "out_features"):
                if key not in e:
                    raise KeyError(f"adapter entry {name!r} has no {key!r}")
            k = int(e["num_gaussians"])
            for key, cols in (("mu_raw", 2), ("chol_raw", 3), ("amp", 1)):
                t = e[key]
                if not isinstance(t, torch.Tensor):
                    raise TypeError(f"{name}.{key}: expected Tensor, got {type(t)!r}")
                if t.shape[0] != k or t.numel() != k * cols:
                    raise ValueError(f"{name}.{key}: shape {tuple(t.shape)} does not hold {k} Gaussians")
            self.shapes.append((int(e["out_features"]), int(e["in_features"]), k))
            mus.append(e["mu_raw"].float().reshape(k, 2))
            chols.append(e["chol_raw"].float().reshape(k, 3))
            amps.append(e["amp"].float().reshape(k, 1))
        self.mu = torch.tanh(torch.cat(mus).to(device)).contiguous()  # on the device, as the layer does
        self.chol_raw = torch.cat(chols).to(device).contiguous()
        self.amp = torch.cat(amps).to(device).contiguous()
        self.n_off = [0]
        for o, i, _ in self.shapes:
            self.n_off.append(self.n_off[-1] + o * i)
        kw = dict(tile_out=int(cfg["tile_out"]), tile_in=int(cfg["tile_in"]),
                  sigma_multiplier=float(cfg["sigma_multiplier"]), normalize=bool(cfg["normalize_gaussian"]),
                  clamp_quad=80.0, out_dtype=out_dtype, out_scale=float(cfg["adapter_scale"]))
        cap_kw, self._measure = _capacity_kw(self.shapes, kw["tile_out"], kw["tile_in"])
        kw.update(cap_kw)
        if base_weights is not None:
            missing = [n for n in self.names if n not in base_weights]
            if missing:
                raise KeyError(f"base_weights lacks {missing}")
            w0 = []
            for n, (o, i, _) in zip(self.names, self.shapes):
                w = base_weights[n]
                if tuple(w.shape) != (o, i):
                    raise ValueError(f"base weight {n!r}: shape {tuple(w.shape)}, expected {(o, i)}")
                w0.append(w.detach().to(device, out_dtype).reshape(-1))
            kw["base_weight"] = torch.cat(w0).contiguous()
        if batch_factory is None:
            from guass_b200.batched import FieldBatch

            def batch_factory(shapes, **k):
                return FieldBatch(shapes, device=device, **k)
        self.batch = batch_factory(self.shapes, **kw)

    @torch.no_grad()
    def render(self) -> dict:
        if self._measure:
            while self.batch.ensure_capacity(self.mu, self.chol_raw, self.amp):
                pass
            self._measure = False
        packed = self.batch.forward(self.mu, self.chol_raw, self.amp)
        return {n: packed[self.n_off[f]:self.n_off[f + 1]].view(o, i)
                for f, (n, (o, i, _)) in enumerate(zip(self.names, self.shapes))}
