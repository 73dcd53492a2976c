"""SD1.5-shaped UNet with Gaussian-field adapters on every attention projection.

The data-parallel training workload of the renderer: a random-init UNet of
the Stable Diffusion 1.5 layout (no checkpoint or dataset is involved), whose
128 attention projections (to_q, to_k, to_v, to_out of 16 transformer
blocks) carry K Gaussian adapters each, trained by epsilon-prediction MSE.
One step renders every adapter's delta through one batched launch set
(:class:`guass_b200.adapters.BatchedAdapters`), runs the UNet forward and
backward, back-propagates the delta gradients through the renderer, all-reduces
the Gaussian-parameter gradients in one flat buffer, and steps the optimizer.

Layout (the SD1.5 UNet): 4 levels of width (320, 640, 1280, 1280), two
residual blocks per level going down and three going up, a transformer block
after each residual block of the first three levels and in the middle block
(self-attention, cross-attention to 77x768 text tokens, GEGLU feed-forward),
8 heads, GroupNorm(32), a 4-channel latent in and out, a sinusoidal timestep
embedding.  :class:`UNetConfig` can shrink every dimension for CPU tests.

Adapter layers (:class:`GaussianProjection`) carry the attributes of GUASS's
``GaussianLinear`` (gaussian_peft/layers/gaussian_linear.py) that the binding
uses -- ``weight`` (frozen), ``bias``, ``mu_raw``, ``chol_raw``, ``amp``,
``adapter_config``, ``compute_delta_weight`` -- and by default apply the delta
the way that layer does (base GEMM plus row-chunked delta GEMMs,
gaussian_linear.py:222-242); ``BatchedAdapters(fused_weight=True)`` replaces
that with one GEMM on W0 + delta.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from guass_b200 import synthetic


@dataclass
class UNetConfig:
    block_channels: tuple = (320, 640, 1280, 1280)
    attn_levels: tuple = (True, True, True, False)
    layers_per_block: int = 2
    heads: int = 8
    cross_dim: int = 768
    text_tokens: int = 77
    latent_channels: int = 4
    latent_size: int = 64
    groups: int = 32
    num_gaussians: int = 256


def tiny_config() -> UNetConfig:
    """A few-MB UNet of the same layout, for CPU tests."""
    return UNetConfig(block_channels=(32, 64), attn_levels=(True, False), layers_per_block=1, heads=2,
                      cross_dim=16, text_tokens=5, latent_size=8, groups=8, num_gaussians=8)


@dataclass
class AdapterSettings:
    """The GaussianAdapterConfig fields the renderer reads
    (gaussian_peft/config/adapter.py)."""
    tile_out: int = 32
    tile_in: int = 32
    sigma_multiplier: float = 3.0
    normalize_gaussian: bool = False
    adapter_scale: float = 1.0


class GaussianProjection(nn.Module):
    """Frozen linear projection plus a Gaussian-field delta (GaussianLinear's
    interface).  Gaussian parameters are drawn with the whole-UNet render
    workload's distributions (log-scale ~ N(log 0.03, 0.5), amp ~ N(0, 1e-3))."""

    def __init__(self, in_features, out_features, bias, k, seed, dtype, settings: AdapterSettings):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.bias = nn.Parameter(torch.zeros(out_features, dtype=dtype), requires_grad=False) if bias else None
        self.adapter_config = settings
        if torch.empty(0).device.type == "meta":  # shapes only (built under torch.device("meta"))
            self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=dtype), requires_grad=False)
            self.mu_raw, self.chol_raw, self.amp = (nn.Parameter(torch.empty(k, c)) for c in (2, 3, 1))
            return
        # seeded on the host (CPU generators), whatever the default device; model.to() moves them
        with torch.device("cpu"):
            g = torch.Generator().manual_seed(10_000 + seed)
            w = torch.randn(out_features, in_features, generator=g) / math.sqrt(in_features)
            f = synthetic.make_field(out_features, in_features, k, seed=seed, log_scale_mean=math.log(0.03),
                                     log_scale_std=0.5)
        self.weight = nn.Parameter(w.to(dtype), requires_grad=False)
        self.mu_raw = nn.Parameter(torch.atanh(f.mu.clamp(-0.999, 0.999)))
        self.chol_raw = nn.Parameter(f.chol_raw.clone())
        self.amp = nn.Parameter(f.amp.clone())

    def compute_delta_weight(self):
        raise RuntimeError("GaussianProjection renders through BatchedAdapters: call install() and render()")

    def forward(self, x):
        # gaussian_linear.py:222-242: base output plus the delta applied in row chunks of max(tile_out, 64)
        delta = self.compute_delta_weight().to(self.weight.dtype)
        out = F.linear(x, self.weight, self.bias)
        rows = min(self.out_features, max(int(self.adapter_config.tile_out), 64))
        parts = [out[..., r:r + rows] + F.linear(x, delta[r:r + rows]) for r in range(0, self.out_features, rows)]
        return torch.cat(parts, dim=-1)


class Attention(nn.Module):
    def __init__(self, dim, ctx_dim, heads, proj):
        super().__init__()
        self.heads = heads
        self.to_q = proj(dim, dim, False)
        self.to_k = proj(ctx_dim, dim, False)
        self.to_v = proj(ctx_dim, dim, False)
        self.to_out = proj(dim, dim, True)

    def forward(self, x, ctx=None):
        ctx = x if ctx is None else ctx
        b, n, d = x.shape
        h = self.heads
        q = self.to_q(x).view(b, n, h, d // h).transpose(1, 2)
        k = self.to_k(ctx).view(b, ctx.shape[1], h, d // h).transpose(1, 2)
        v = self.to_v(ctx).view(b, ctx.shape[1], h, d // h).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v)
        return self.to_out(o.transpose(1, 2).reshape(b, n, d))


class TransformerBlock(nn.Module):
    def __init__(self, ch, cfg: UNetConfig, proj):
        super().__init__()
        self.norm = nn.GroupNorm(cfg.groups, ch, eps=1e-6)
        self.proj_in = nn.Conv2d(ch, ch, 1)
        self.norm1, self.norm2, self.norm3 = nn.LayerNorm(ch), nn.LayerNorm(ch), nn.LayerNorm(ch)
        self.attn1 = Attention(ch, ch, cfg.heads, proj)
        self.attn2 = Attention(ch, cfg.cross_dim, cfg.heads, proj)
        self.ff_in = nn.Linear(ch, 8 * ch)   # GEGLU: value and gate halves
        self.ff_out = nn.Linear(4 * ch, ch)
        self.proj_out = nn.Conv2d(ch, ch, 1)

    def forward(self, x, ctx):
        b, c, hh, ww = x.shape
        res = x
        t = self.proj_in(self.norm(x)).flatten(2).transpose(1, 2)
        t = t + self.attn1(self.norm1(t))
        t = t + self.attn2(self.norm2(t), ctx)
        a, gate = self.ff_in(self.norm3(t)).chunk(2, dim=-1)
        t = t + self.ff_out(a * F.gelu(gate))
        return self.proj_out(t.transpose(1, 2).reshape(b, c, hh, ww)) + res


class ResBlock(nn.Module):
    def __init__(self, cin, cout, tdim, groups):
        super().__init__()
        self.norm1 = nn.GroupNorm(groups, cin, eps=1e-5)
        self.conv1 = nn.Conv2d(cin, cout, 3, padding=1)
        self.temb = nn.Linear(tdim, cout)
        self.norm2 = nn.GroupNorm(groups, cout, eps=1e-5)
        self.conv2 = nn.Conv2d(cout, cout, 3, padding=1)
        self.skip = nn.Conv2d(cin, cout, 1) if cin != cout else nn.Identity()

    def forward(self, x, temb):
        h = self.conv1(F.silu(self.norm1(x)))
        h = h + self.temb(F.silu(temb))[:, :, None, None]
        h = self.conv2(F.silu(self.norm2(h)))
        return h + self.skip(x)


def timestep_embedding(t, dim):
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    args = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


class SD15UNet(nn.Module):
    """The UNet; ``adapters()`` lists its GaussianProjection layers by name."""

    def __init__(self, cfg: UNetConfig = UNetConfig(), dtype=torch.bfloat16, settings: AdapterSettings | None = None):
        super().__init__()
        self.cfg = cfg
        settings = settings or AdapterSettings()
        counter = [0]

        def proj(i, o, bias):
            counter[0] += 1
            return GaussianProjection(i, o, bias, cfg.num_gaussians, counter[0], dtype, settings)

        chs = cfg.block_channels
        c0, tdim = chs[0], 4 * chs[0]
        self.conv_in = nn.Conv2d(cfg.latent_channels, c0, 3, padding=1)
        self.time1, self.time2 = nn.Linear(c0, tdim), nn.Linear(tdim, tdim)
        self.down = nn.ModuleList()
        skips, ch = [c0], c0
        for i, c in enumerate(chs):
            level = nn.ModuleList()
            for _ in range(cfg.layers_per_block):
                level.append(ResBlock(ch, c, tdim, cfg.groups))
                ch = c
                if cfg.attn_levels[i]:
                    level.append(TransformerBlock(ch, cfg, proj))
                skips.append(ch)
            if i != len(chs) - 1:
                level.append(nn.Conv2d(ch, ch, 3, stride=2, padding=1))
                skips.append(ch)
            self.down.append(level)
        self.mid = nn.ModuleList([ResBlock(ch, ch, tdim, cfg.groups), TransformerBlock(ch, cfg, proj),
                                  ResBlock(ch, ch, tdim, cfg.groups)])
        self.up = nn.ModuleList()
        for i in reversed(range(len(chs))):
            c = chs[i]
            level = nn.ModuleList()
            for _ in range(cfg.layers_per_block + 1):
                level.append(ResBlock(ch + skips.pop(), c, tdim, cfg.groups))
                ch = c
                if cfg.attn_levels[i]:
                    level.append(TransformerBlock(ch, cfg, proj))
            if i != 0:
                level.append(nn.Conv2d(ch, ch, 3, padding=1))  # after a nearest x2 upsample
            self.up.append(level)
        self.norm_out = nn.GroupNorm(cfg.groups, ch, eps=1e-5)
        self.conv_out = nn.Conv2d(ch, cfg.latent_channels, 3, padding=1)
        for name, p in self.named_parameters():
            if not name.endswith(("mu_raw", "chol_raw", "amp")):
                p.requires_grad_(False)
                p.data = p.data.to(dtype)

    def adapters(self) -> dict:
        return {n: m for n, m in self.named_modules() if isinstance(m, GaussianProjection)}

    def forward(self, x, t, ctx):
        temb = self.time2(F.silu(self.time1(timestep_embedding(t, self.cfg.block_channels[0]).to(x.dtype))))
        h = self.conv_in(x)
        skips = [h]
        for i, level in enumerate(self.down):
            for blk in level:
                if isinstance(blk, ResBlock):
                    h = blk(h, temb)
                    if not self.cfg.attn_levels[i]:
                        skips.append(h)
                elif isinstance(blk, TransformerBlock):
                    h = blk(h, ctx)
                    skips.append(h)
                else:  # downsample
                    h = blk(h)
                    skips.append(h)
        h = self.mid[2](self.mid[1](self.mid[0](h, temb), ctx), temb)
        for level in self.up:
            for blk in level:
                if isinstance(blk, ResBlock):
                    h = blk(torch.cat([h, skips.pop()], dim=1), temb)
                elif isinstance(blk, TransformerBlock):
                    h = blk(h, ctx)
                else:  # upsample
                    h = blk(F.interpolate(h, scale_factor=2.0, mode="nearest"))
        return self.conv_out(F.silu(self.norm_out(h)))


def noise_schedule(device, steps: int = 1000):
    """alphas_cumprod of the SD1.5 "scaled_linear" beta schedule (0.00085 .. 0.012)."""
    betas = torch.linspace(0.00085 ** 0.5, 0.012 ** 0.5, steps, dtype=torch.float64) ** 2
    return torch.cumprod(1.0 - betas, 0).to(device=device, dtype=torch.float32)


@dataclass
class StepInputs:
    latents: torch.Tensor   # [B, 4, S, S]
    text: torch.Tensor      # [B, T, cross_dim]
    t: torch.Tensor         # [B] int64 in [0, 1000)
    noise: torch.Tensor     # [B, 4, S, S] epsilon
    fields: list = field(default_factory=list)

    def tensors(self):
        return [self.latents, self.text, self.t, self.noise]


def synthetic_inputs(cfg: UNetConfig, batch: int, seed: int, device="cpu", dtype=torch.bfloat16) -> StepInputs:
    """Per-rank inputs: latents and text ~ N(0, 1), t ~ U{0..999}, noise ~ N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    s = cfg.latent_size
    return StepInputs(
        latents=torch.randn(batch, cfg.latent_channels, s, s, generator=g).to(device, dtype),
        text=torch.randn(batch, cfg.text_tokens, cfg.cross_dim, generator=g).to(device, dtype),
        t=torch.randint(0, 1000, (batch,), generator=g).to(device),
        noise=torch.randn(batch, cfg.latent_channels, s, s, generator=g).to(device, dtype),
    )


def diffusion_loss(model: SD15UNet, inp: StepInputs, alphas_cumprod) -> torch.Tensor:
    """Epsilon-prediction MSE at the sampled timesteps (fp32 loss)."""
    ab = alphas_cumprod[inp.t].view(-1, 1, 1, 1)
    x_t = (ab.sqrt() * inp.latents.float() + (1 - ab).sqrt() * inp.noise.float()).to(inp.latents.dtype)
    pred = model(x_t, inp.t, inp.text)
    return F.mse_loss(pred.float(), inp.noise.float())


class PerLayerRender:
    """The reference's call pattern: every GaussianProjection renders its own
    delta inside its forward through the drop-in runtime
    (``guass_b200.cuda_field.gaussian_field_train``, i.e. what
    GaussianLinear.compute_delta_weight does in ``cuda_field_train`` mode,
    gaussian_linear.py:178-197): one render and one backward per layer.
    ``render()`` is a no-op so that it can stand in for
    :class:`~guass_b200.adapters.BatchedAdapters` in :class:`DataParallelTrainer`."""

    def __init__(self, modules: dict):
        self.modules = list(modules.values())
        self._orig = {}

    def install(self):
        from guass_b200.cuda_field import gaussian_field_train

        for m in self.modules:
            if id(m) in self._orig:
                continue
            self._orig[id(m)] = m.compute_delta_weight
            dev = m.mu_raw.device
            rows = torch.linspace(-1.0, 1.0, m.out_features, device=dev)
            cols = torch.linspace(-1.0, 1.0, m.in_features, device=dev)

            def cdw(m=m, rows=rows, cols=cols):
                c = m.adapter_config
                delta = gaussian_field_train(row_coords=rows, col_coords=cols, mu=torch.tanh(m.mu_raw),
                                             chol_raw=m.chol_raw, amp=m.amp, tile_out=c.tile_out, tile_in=c.tile_in,
                                             sigma_multiplier=c.sigma_multiplier, normalize=c.normalize_gaussian,
                                             clamp_quad=80.0)
                return delta.view(m.out_features, m.in_features) * c.adapter_scale

            m.compute_delta_weight = cdw

    def render(self):
        return None


class DataParallelTrainer:
    """One data-parallel training step of the adapters (one process per GPU).

    ``step(inputs)``: render every delta (one batched launch set), UNet
    forward + epsilon MSE, backward (the renderer's batched backward gives the
    Gaussian-parameter gradients), one flat all-reduce of those gradients
    averaged over the ranks (:func:`guass_b200.adapters.allreduce_adapter_grads`),
    AdamW step.  Returns the detached loss."""

    def __init__(self, model: SD15UNet, bank, lr: float = 1e-4, world: int = 1, group=None):
        from guass_b200.adapters import adapter_parameters

        self.model, self.bank, self.world, self.group = model, bank, world, group
        self.mods = list(model.adapters().values())
        self.params = adapter_parameters(self.mods)
        self.opt = torch.optim.AdamW(self.params, lr=lr)
        self.alphas_cumprod = noise_schedule(self.params[0].device)
        # optional list of (start, end) CUDA events around each step's all-reduce
        self.allreduce_events = None

    def backward(self, inputs: StepInputs) -> torch.Tensor:
        """Render, forward, backward and gradient all-reduce (no optimizer step)."""
        from guass_b200.adapters import allreduce_adapter_grads

        self.bank.render()
        loss = diffusion_loss(self.model, inputs, self.alphas_cumprod)
        loss.backward()
        if self.world > 1:
            ev = None
            if self.allreduce_events is not None:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            allreduce_adapter_grads(self.mods, group=self.group)
            if ev is not None:
                ev[1].record()
                self.allreduce_events.append(ev)
        return loss.detach()

    def step(self, inputs: StepInputs) -> torch.Tensor:
        loss = self.backward(inputs)
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss
