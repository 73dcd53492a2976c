"""Densify statistics kernel (gf_grad_stats_accumulate via
guass_b200.stats.BatchedStatsTracker) against a plain PyTorch fp32
restatement of GaussianStatsTracker (gaussian_peft/controllers/stats.py:47-131).

contrib and active_steps are fp32 adds of the same numbers, so they must be
equal; the gradient norms (torch's reduction for the reference, one fma
chain here) may differ by an ulp, so they are held to 1e-6 relative."""
from __future__ import annotations

import pytest
import torch
from torch import nn

from guass_b200.stats import BatchedStatsTracker

pytestmark = pytest.mark.gpu


def _torch_scores(steps):
    """steps: list of (mu_g, chol_g, amp_g, amp) -> reference scores (stats.py)."""
    def score(g):
        if g is None:
            return None
        g = g.detach().float()
        return torch.linalg.vector_norm(g.reshape(g.shape[0], -1), dim=1).reshape(-1, 1)

    acc = None
    for mu_g, chol_g, amp_g, amp in steps:
        k = amp.shape[0]
        if acc is None:
            acc = [torch.zeros(k, 1, device=amp.device) for _ in range(5)]
        for i, g in enumerate((mu_g, chol_g, amp_g)):
            s = score(g)
            if s is not None:
                acc[i].add_(s)
        acc[3].add_(amp.detach().float().reshape(k, -1).abs().mean(dim=1).reshape(-1, 1))
        acc[4].add_(1.0)
    active = acc[4].clamp_min(1.0)
    return {"grad_mu": acc[0] / active, "grad_cov": acc[1] / active, "grad_amp": acc[2] / active,
            "grad_score": (acc[0] + acc[1] + acc[2]) / active, "contrib_score": acc[3] / active,
            "active_steps": acc[4]}


class _Layer(nn.Module):
    def __init__(self, k):
        super().__init__()
        self.mu_raw = nn.Parameter(torch.zeros(k, 2, device="cuda"))
        self.chol_raw = nn.Parameter(torch.zeros(k, 3, device="cuda"))
        self.amp = nn.Parameter(torch.zeros(k, 1, device="cuda"))


def test_update_from_model_matches_torch_restatement():
    ks = [256, 1, 1000, 37, 4096]
    model = nn.ModuleDict({f"l{i}": _Layer(k) for i, k in enumerate(ks)})
    tracker = BatchedStatsTracker()
    history = {n: [] for n in model}
    gen = torch.Generator(device="cuda").manual_seed(0)
    for step in range(3):
        for n, m in model.items():
            with torch.no_grad():
                m.amp.copy_(torch.randn(m.amp.shape, generator=gen, device="cuda") * 1e-3)
            for p in (m.mu_raw, m.chol_raw, m.amp):
                p.grad = torch.randn(p.shape, generator=gen, device="cuda") * 10.0 ** (-step)
            if n == "l3":
                m.chol_raw.grad = None  # a parameter without a gradient adds nothing
            history[n].append((m.mu_raw.grad, m.chol_raw.grad, m.amp.grad, m.amp.detach().clone()))
        tracker.update_from_model(model)
    for n in model:
        got, want = tracker.get_scores(n), _torch_scores(history[n])
        for key in ("contrib_score", "active_steps"):
            assert torch.equal(got[key], want[key]), (n, key)
        for key in ("grad_mu", "grad_cov", "grad_amp", "grad_score"):
            torch.testing.assert_close(got[key], want[key], rtol=1e-6, atol=0, msg=f"{n}:{key}")
    tracker.reset_all()
    assert not tracker.get_scores("l0")["active_steps"].any()


def test_layer_update_converts_dtype_and_checks_shapes():
    tracker = BatchedStatsTracker()
    tracker.register_layer("a", 64, "cuda")
    g = torch.randn(64, 2, device="cuda", dtype=torch.bfloat16)
    tracker.update_from_layer_grads("a", g, None, None)
    want = torch.linalg.vector_norm(g.float(), dim=1).reshape(-1, 1)
    torch.testing.assert_close(tracker.get_scores("a")["grad_mu"], want, rtol=1e-6, atol=0)
    with pytest.raises(RuntimeError, match="expected 64x3"):
        tracker.update_from_layer_grads("a", None, torch.zeros(64, 2, device="cuda"), None)
