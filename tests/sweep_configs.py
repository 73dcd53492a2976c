"""Seeded random render configurations shared by the oracle-vs-reference
sweep (CPU) and the CUDA-vs-oracle sweep (GPU): the same seeds give the same
fields and settings in both."""
from __future__ import annotations

import math

import numpy as np

from guass_b200.synthetic import make_field


def draw(seed: int):
    """(field, dict(tile_out, tile_in, sigma_multiplier, normalize, clamp_quad))."""
    rng = np.random.default_rng(1000 + seed)
    out_f, in_f = int(rng.integers(1, 130)), int(rng.integers(1, 130))
    k = int(rng.integers(1, 40))
    to, ti = int(rng.choice([8, 16, 32, 13, 64])), int(rng.choice([8, 16, 32, 7, 64]))
    sigma = float(rng.choice([1.5, 2.0, 3.0, 4.5]))
    norm = bool(rng.integers(0, 2))
    clamp = [80.0, None, 20.0][int(rng.integers(0, 3))]
    f = make_field(out_f, in_f, k, seed=seed, log_scale_mean=math.log(float(rng.choice([0.03, 0.1, 0.3]))),
                   log_scale_std=0.6, elongated_frac=float(rng.choice([0.0, 0.5])))
    return f, dict(tile_out=to, tile_in=ti, sigma_multiplier=sigma, normalize=norm, clamp_quad=clamp)
