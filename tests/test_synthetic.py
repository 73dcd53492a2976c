"""Seeded synthetic inputs with the benchmark configurations' shapes."""
from __future__ import annotations

import torch

from guass_b200 import synthetic as S


def test_seeded_and_deterministic():
    a, b = S.cfg1(0), S.cfg1(0)
    for x, y in zip((a.mu, a.chol_raw, a.amp, a.grad), (b.mu, b.chol_raw, b.amp, b.grad)):
        assert torch.equal(x, y)
    assert not torch.equal(S.cfg1(1).mu, a.mu)


def test_config_shapes():
    c0, c1, c2 = S.cfg0(), S.cfg1(), S.cfg2()
    assert (c0.out_features, c0.in_features, c0.k) == (320, 320, 64)
    assert (c1.out_features, c1.in_features, c1.k) == (320, 768, 256)
    assert (c2.out_features, c2.in_features, c2.k) == (1280, 1280, 1024)
    for c in (c0, c1, c2):
        assert c.mu.dtype == torch.float32 and c.mu.shape == (c.k, 2)
        assert c.chol_raw.shape == (c.k, 3) and c.amp.shape == (c.k, 1)
        assert c.grad.numel() == c.numel
        assert float(c.mu.abs().max()) <= 1.0


def test_unet_projection_shapes():
    shapes = S.unet_projection_shapes()
    assert len(shapes) == 128
    assert sum(o * i for _, o, i in shapes) == 93_511_680
    widths = sorted({o for _, o, _ in shapes})
    assert widths == [320, 640, 1280]


def test_parameter_mapping_reproduces_covariance():
    # Sigma = L L^T with L from chol_raw must equal R diag(s^2) R^T
    import math
    u = torch.tensor([[0.5, 0.5]], dtype=torch.float64)
    log_s = torch.tensor([[math.log(0.05), math.log(0.01)]], dtype=torch.float64)
    theta = torch.tensor([0.7], dtype=torch.float64)
    mu, chol_raw, amp = S.params_from_normalised(u, log_s, theta, torch.tensor([1e-3], dtype=torch.float64))
    sp = torch.nn.functional.softplus
    r = chol_raw.double()[0]
    L = torch.tensor([[sp(r[0]) + 1e-5, 0.0], [r[1], sp(r[2]) + 1e-5]], dtype=torch.float64)
    s = 2 * torch.exp(log_s[0])
    R = torch.tensor([[math.cos(0.7), -math.sin(0.7)], [math.sin(0.7), math.cos(0.7)]], dtype=torch.float64)
    want = R @ torch.diag(s * s) @ R.T
    assert torch.allclose(L @ L.T, want, rtol=1e-5, atol=1e-9)
    assert torch.allclose(mu, torch.zeros(1, 2))
