"""Seeded synthetic Gaussian fields with the BASELINE configurations' shapes.

No dataset is involved in this path: every input is drawn here from a seeded
``torch.Generator`` on the CPU, so a config and a seed name one exact input.

Distributions are drawn in the normalised [0, 1]^2 matrix space that the
benchmark configurations are stated in (mean, per-axis log-scale, rotation,
amplitude) and converted once to the renderer's parameterisation:

* ``mu = 2u - 1`` (the renderer's axes are ``linspace(-1, 1)``,
  gaussian_peft/kernels/coords.py:23-34),
* ``s_ref = 2 s``, ``Sigma = R diag(s_ref^2) R^T``, ``L = chol(Sigma)``,
* ``chol_raw = (softplus^-1(L00 - eps), L10, softplus^-1(L11 - eps))`` with
  ``eps = 1e-5`` (gaussian_peft/cuda_field/csrc/forward.cu:163-171).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

CHOLESKY_EPS = 1e-5


@dataclass
class FieldInputs:
    """One Gaussian field: the reference forward's inputs plus an upstream grad."""

    out_features: int
    in_features: int
    row_coords: torch.Tensor  # [out] f32
    col_coords: torch.Tensor  # [in] f32
    mu: torch.Tensor  # [K, 2] f32
    chol_raw: torch.Tensor  # [K, 3] f32
    amp: torch.Tensor  # [K, 1] f32
    grad: torch.Tensor  # [out*in] f32, dL/dDeltaW
    name: str = ""

    @property
    def k(self) -> int:
        return int(self.mu.shape[0])

    @property
    def numel(self) -> int:
        return self.out_features * self.in_features

    def to(self, device) -> "FieldInputs":
        return FieldInputs(
            self.out_features, self.in_features,
            *(t.to(device) for t in (self.row_coords, self.col_coords, self.mu,
                                     self.chol_raw, self.amp, self.grad)),
            name=self.name,
        )


def _inv_softplus(y: torch.Tensor) -> torch.Tensor:
    # log(expm1(y)), stable for small and large y
    return torch.where(y > 20.0, y, torch.log(torch.expm1(y)))


def params_from_normalised(u: torch.Tensor, log_s: torch.Tensor, theta: torch.Tensor,
                           amp: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(mean in [0,1]^2, per-axis log-scale, rotation, amp) -> (mu, chol_raw, amp[K,1])."""
    u = u.double()
    s = 2.0 * torch.exp(log_s.double())  # s_ref = 2 s
    c, sn = torch.cos(theta.double()), torch.sin(theta.double())
    s0sq, s1sq = s[:, 0] ** 2, s[:, 1] ** 2
    sig00 = c * c * s0sq + sn * sn * s1sq
    sig01 = c * sn * (s0sq - s1sq)
    sig11 = sn * sn * s0sq + c * c * s1sq
    l00 = torch.sqrt(sig00)
    l10 = sig01 / l00
    l11 = torch.sqrt(torch.clamp(sig11 - l10 * l10, min=1e-12))
    raw0 = _inv_softplus(torch.clamp(l00 - CHOLESKY_EPS, min=1e-7))
    raw2 = _inv_softplus(torch.clamp(l11 - CHOLESKY_EPS, min=1e-7))
    chol_raw = torch.stack([raw0, l10, raw2], dim=1).float().contiguous()
    mu = (2.0 * u - 1.0).float().contiguous()
    return mu, chol_raw, amp.reshape(-1, 1).float().contiguous()


def _axes(out_features: int, in_features: int) -> tuple[torch.Tensor, torch.Tensor]:
    # gaussian_peft/kernels/coords.py:37-50 (build_linear_axes)
    return (torch.linspace(-1.0, 1.0, out_features, dtype=torch.float32),
            torch.linspace(-1.0, 1.0, in_features, dtype=torch.float32))


def make_field(out_features: int, in_features: int, k: int, *, seed: int = 0,
               log_scale_mean: float = math.log(0.05), log_scale_std: float = 0.3,
               amp_std: float = 1e-3, grad_std: float = 1.0, elongated_frac: float = 0.0,
               elongation: tuple[float, float] = (5.0, 20.0), blob_frac: float = 0.0,
               num_blobs: int = 8, blob_std: float = 0.05, name: str = "") -> FieldInputs:
    """Draw one field.  See the module docstring for the parameter mapping."""
    g = torch.Generator().manual_seed(seed)
    u = torch.rand(k, 2, generator=g, dtype=torch.float64)
    n_blob = int(round(blob_frac * k))
    if n_blob:
        centres = torch.rand(num_blobs, 2, generator=g, dtype=torch.float64) * 0.8 + 0.1
        which = torch.randint(0, num_blobs, (n_blob,), generator=g)
        pts = centres[which] + blob_std * torch.randn(n_blob, 2, generator=g, dtype=torch.float64)
        u[:n_blob] = pts.clamp(0.0, 1.0)
    log_s = log_scale_mean + log_scale_std * torch.randn(k, 2, generator=g, dtype=torch.float64)
    theta = (torch.rand(k, generator=g, dtype=torch.float64) * 2.0 - 1.0) * math.pi
    n_el = int(round(elongated_frac * k))
    if elongated_frac > 0.0:
        # isotropic majority: one scale for both axes
        log_s[:, 1] = log_s[:, 0]
        if n_el:
            ratio = elongation[0] + (elongation[1] - elongation[0]) * torch.rand(
                n_el, generator=g, dtype=torch.float64)
            # major axis keeps the drawn scale, minor axis = scale / ratio
            idx = torch.arange(k - n_el, k)
            log_s[idx, 1] = log_s[idx, 0] - torch.log(ratio)
    amp = amp_std * torch.randn(k, generator=g, dtype=torch.float64)
    mu, chol_raw, amp_t = params_from_normalised(u, log_s, theta, amp)
    row, col = _axes(out_features, in_features)
    grad = (grad_std * torch.randn(out_features * in_features, generator=g, dtype=torch.float64)).float()
    return FieldInputs(out_features, in_features, row, col, mu, chol_raw, amp_t, grad, name=name)


def cfg0(seed: int = 0) -> FieldInputs:
    """320x320, K=64, log s ~ N(log .05, .3), amp ~ N(0, 1e-3), g ~ N(0, 1)."""
    return make_field(320, 320, 64, seed=seed, name="cfg0")


def cfg1(seed: int = 0) -> FieldInputs:
    """Cross-attention to_k: 320x768, K=256, log s ~ N(log .03, .5), g ~ N(0, 1e-2)."""
    return make_field(320, 768, 256, seed=seed, log_scale_mean=math.log(0.03), log_scale_std=0.5,
                      grad_std=1e-2, name="cfg1")


def cfg2(seed: int = 0) -> FieldInputs:
    """1280x1280, K=1024: 75% isotropic (log s ~ N(log .02, .3)), 25% elongated 5-20x,
    half the means in 8 blobs of sigma .05."""
    return make_field(1280, 1280, 1024, seed=seed, log_scale_mean=math.log(0.02), log_scale_std=0.3,
                      elongated_frac=0.25, blob_frac=0.5, name="cfg2")


def unet_projection_shapes() -> list[tuple[str, int, int]]:
    """SD1.5 UNet attention projections: 16 transformer blocks (5 at width 320,
    5 at 640, 6 at 1280); attn1 q/k/v/out are d x d, attn2 q/out are d x d and
    attn2 k/v are d x 768.  Returns (name, out_features, in_features), 128 rows."""
    widths = [320, 320, 640, 640, 1280, 1280, 1280, 1280, 1280, 1280, 640, 640, 640, 320, 320, 320]
    names = (["down"] * 6) + ["mid"] + (["up"] * 9)
    shapes = []
    for b, (d, part) in enumerate(zip(widths, names)):
        for proj in ("to_q", "to_k", "to_v", "to_out"):
            shapes.append((f"{part}{b}.attn1.{proj}", d, d))
        for proj in ("to_q", "to_k", "to_v", "to_out"):
            in_f = 768 if proj in ("to_k", "to_v") else d
            shapes.append((f"{part}{b}.attn2.{proj}", d, in_f))
    return shapes


def cfg3(seed: int = 0, k: int = 256) -> list[FieldInputs]:
    """Whole-UNet batch: 128 projections, K=256 each, cfg1's distributions."""
    fields = []
    for i, (name, out_f, in_f) in enumerate(unet_projection_shapes()):
        fields.append(make_field(out_f, in_f, k, seed=seed * 1000 + i, log_scale_mean=math.log(0.03),
                                 log_scale_std=0.5, grad_std=1e-2, name=name))
    return fields


def densified(k: int, seed: int = 0) -> FieldInputs:
    """A 1280x1280 field after densification (gaussian_peft/trainers/
    base_trainer.py:127-220 clones and splits Gaussians, so K grows while each
    one shrinks): K Gaussians with log s ~ N(log(0.02 * sqrt(1024 / K)), 0.3)
    (the covered area stays about that of cfg2's K=1024), 25% elongated, half
    the means in 8 blobs as cfg2."""
    return make_field(1280, 1280, k, seed=seed, log_scale_mean=math.log(0.02 * math.sqrt(1024.0 / k)),
                      log_scale_std=0.3, elongated_frac=0.25, blob_frac=0.5, name=f"dense{k}")


def degenerate_scan(k: int, out_f: int = 1280, in_f: int = 1280) -> FieldInputs:
    """K tiny Gaussians all inside the first tile of a field: every other tile
    has no pair, so a render of it costs the per-tile candidate scan over the
    K boxes (plus one tile's K x 1024 evaluations) -- an upper bound on the
    scan's share of a real render with the same K."""
    f = make_field(out_f, in_f, k, seed=7, log_scale_mean=math.log(1e-4), log_scale_std=0.1)
    f.mu[:, 0] = -1.0 + 1.0 / out_f
    f.mu[:, 1] = -1.0 + 1.0 / in_f
    return f


CONFIGS = {"cfg0": cfg0, "cfg1": cfg1, "cfg2": cfg2}
