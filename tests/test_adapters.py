"""Whole-model adapter plumbing (guass_b200.adapters), on the CPU.

The batch is a test double computed with the CPU oracle, so these tests check
the autograd wiring, the module binding, the flat gradient all-reduce (gloo
ranks) and the checkpoint format -- not the CUDA kernels, which the GPU tests
cover through the same FieldBatch interface.
"""
from __future__ import annotations

import math
import os
import socket
from dataclasses import dataclass

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F
from torch import nn

import oracle
from guass_b200 import synthetic
from oracle_batch import OracleBatch
from guass_b200.adapters import (BatchedAdapters, CheckpointFields, adapter_state_dict, allreduce_adapter_grads,
                                 load_adapter_state_dict)


@dataclass
class Cfg:
    tile_out: int = 32
    tile_in: int = 32
    sigma_multiplier: float = 3.0
    normalize_gaussian: bool = False
    adapter_scale: float = 1.0


class FakeLinear(nn.Module):
    """The attributes of GaussianLinear that the binding uses."""

    def __init__(self, out_f, in_f, k, seed, scale=1.0):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(out_f, in_f, generator=torch.Generator().manual_seed(seed)),
                                   requires_grad=False)
        f = synthetic.make_field(out_f, in_f, k, seed=seed, log_scale_mean=math.log(0.08))
        self.out_features, self.in_features = out_f, in_f
        self.mu_raw = nn.Parameter(torch.atanh(f.mu.clamp(-0.999, 0.999)))
        self.chol_raw = nn.Parameter(f.chol_raw.clone())
        self.amp = nn.Parameter(f.amp.clone())
        self.row_coords, self.col_coords = f.row_coords, f.col_coords
        self.adapter_config = Cfg(adapter_scale=scale)
        self.bias = None

    def compute_delta_weight(self):
        raise AssertionError("the binding must replace this")


def _modules():
    return {"a": FakeLinear(40, 70, 6, 1), "b": FakeLinear(64, 32, 9, 2, scale=0.5), "c": FakeLinear(33, 40, 4, 3)}


def test_render_matches_per_field_oracle_and_binds_modules():
    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    deltas = bank.render()
    for (name, m), d in zip(mods.items(), deltas):
        want, _, _ = oracle.forward(m.row_coords, m.col_coords, torch.tanh(m.mu_raw).detach(), m.chol_raw.detach(),
                                    m.amp.detach())
        assert torch.allclose(d, torch.from_numpy(want).view(m.out_features, m.in_features)
                              * m.adapter_config.adapter_scale)
    bank.install()
    for m, d in zip(mods.values(), deltas):
        assert m.compute_delta_weight() is d
    bank.uninstall()
    with pytest.raises(AssertionError):
        mods["a"].compute_delta_weight()


def test_gradients_reach_module_parameters():
    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    gs = [torch.randn(m.out_features, m.in_features, generator=torch.Generator().manual_seed(i))
          for i, m in enumerate(mods.values())]
    loss = sum((d * g).sum() for d, g in zip(bank.render(), gs))
    loss.backward()
    for m, g in zip(mods.values(), gs):
        mu = torch.tanh(m.mu_raw).detach()
        _, tp, ids = oracle.forward(m.row_coords, m.col_coords, mu, m.chol_raw.detach(), m.amp.detach())
        d_mu, d_chol, d_amp = oracle.backward((g * m.adapter_config.adapter_scale).reshape(-1), m.row_coords,
                                              m.col_coords, mu, m.chol_raw.detach(), m.amp.detach(), tp, ids)
        assert torch.allclose(m.mu_raw.grad, torch.from_numpy(d_mu) * (1 - mu * mu), rtol=1e-5, atol=1e-9)
        assert torch.allclose(m.chol_raw.grad, torch.from_numpy(d_chol), rtol=1e-5, atol=1e-9)
        assert torch.allclose(m.amp.grad, torch.from_numpy(d_amp), rtol=1e-5, atol=1e-9)


def test_mixed_render_settings_rejected():
    mods = _modules()
    mods["b"].adapter_config = Cfg(tile_out=16)
    with pytest.raises(ValueError, match="share tile size"):
        BatchedAdapters(mods, batch_factory=OracleBatch)


def test_adapter_checkpoint_roundtrip_and_schema(tmp_path):
    mods = _modules()
    state = adapter_state_dict(mods)
    assert set(state["a"]) == {"mu_raw", "chol_raw", "amp", "num_gaussians", "in_features", "out_features",
                               "has_bias"}
    path = tmp_path / "adapter.pt"
    torch.save({"format": "gaussian-peft-adapter", "step": 3, "adapters": state}, path)
    other = _modules()
    for m in other.values():
        with torch.no_grad():
            m.amp.zero_()
    load_adapter_state_dict(other, torch.load(path)["adapters"])
    for n in mods:
        assert torch.equal(other[n].amp, mods[n].amp) and torch.equal(other[n].mu_raw, mods[n].mu_raw)
    bad = dict(state)
    bad["a"] = dict(state["a"], in_features=71)
    with pytest.raises(ValueError, match="schema mismatch"):
        load_adapter_state_dict(other, bad)
    with pytest.raises(KeyError):
        load_adapter_state_dict(other, {"zzz": state["a"]})


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mods = _modules()
        for m in mods.values():  # rank-dependent gradients
            for p in (m.mu_raw, m.chol_raw, m.amp):
                p.grad = torch.full_like(p, float(rank + 1))
        allreduce_adapter_grads(mods.values())
        ok = all(bool((p.grad == 1.5).all()) for m in mods.values() for p in (m.mu_raw, m.chol_raw, m.amp))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_flat_allreduce_on_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert dict(q.get(timeout=10) for _ in procs) == {0: True, 1: True}


def test_consecutive_steps_render_and_backward():
    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    opt = torch.optim.SGD([p for m in mods.values() for p in (m.mu_raw, m.chol_raw, m.amp)], lr=1e-3)
    first = None
    for step in range(2):
        opt.zero_grad()
        loss = sum(d.square().sum() for d in bank.render())
        loss.backward()
        g = mods["b"].amp.grad.clone()
        if first is None:
            first = g
        opt.step()
    assert bank.batch.calls == 2
    assert not torch.equal(first, g)  # parameters moved, gradients follow


def test_freeze_serves_cached_render():
    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    bank.install()
    frozen = bank.freeze()
    calls = bank.batch.calls
    for _ in range(3):  # e.g. denoising steps
        assert all(torch.equal(m.compute_delta_weight(), d) for m, d in zip(mods.values(), frozen))
        bank.render()
    assert bank.batch.calls == calls
    bank.unfreeze()
    bank.render()
    assert bank.batch.calls == calls + 1


def test_densify_rebuild():
    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    bank.install()
    assert not bank.shapes_changed()
    m = mods["b"]  # clone two Gaussians, like densify
    m.mu_raw = nn.Parameter(torch.cat([m.mu_raw.detach(), m.mu_raw.detach()[:2]]))
    m.chol_raw = nn.Parameter(torch.cat([m.chol_raw.detach(), m.chol_raw.detach()[:2]]))
    m.amp = nn.Parameter(torch.cat([m.amp.detach(), m.amp.detach()[:2]]))
    assert bank.shapes_changed()
    bank = bank.rebuilt()
    assert bank.shapes[1][2] == 11 and not bank.shapes_changed()
    deltas = bank.render()
    assert torch.equal(mods["b"].compute_delta_weight(), deltas[1])


def _grads(mods):
    return [p.grad.clone() for m in mods.values() for p in (m.mu_raw, m.chol_raw, m.amp)]


def test_fused_weight_equals_base_plus_delta_gemms():
    """One GEMM with W0 + s*delta gives the reference layer's output
    (F.linear(x, W0) + F.linear(x, s*delta), gaussian_linear.py:222-242) and
    the same adapter gradients."""
    def make():
        return {"a": FakeLinear(40, 70, 6, 1, scale=0.5), "b": FakeLinear(64, 32, 9, 2, scale=0.5)}

    gen = torch.Generator().manual_seed(3)
    xs = {"a": torch.randn(5, 70, generator=gen), "b": torch.randn(5, 32, generator=gen)}
    gys = {"a": torch.randn(5, 40, generator=gen), "b": torch.randn(5, 64, generator=gen)}

    plain = make()
    bank = BatchedAdapters(plain, batch_factory=OracleBatch, out_dtype=torch.float32)
    bank.install()
    bank.render()
    ref_y = {n: F.linear(xs[n], m.weight) + F.linear(xs[n], m.compute_delta_weight()) for n, m in plain.items()}
    sum((ref_y[n] * gys[n]).sum() for n in plain).backward()

    fused = make()
    fbank = BatchedAdapters(fused, batch_factory=OracleBatch, out_dtype=torch.float32, fused_weight=True)
    fbank.install()
    fbank.render()
    y = {n: m(xs[n]) for n, m in fused.items()}
    sum((y[n] * gys[n]).sum() for n in fused).backward()
    for n in plain:
        torch.testing.assert_close(y[n], ref_y[n], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(fused[n].compute_delta_weight(), plain[n].compute_delta_weight().detach(),
                                   rtol=0, atol=1e-6)  # W_eff - W0 keeps an ulp of |W0| <= ~4
    for a, b in zip(_grads(fused), _grads(plain)):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-9)
    fbank.uninstall()
    with pytest.raises(NotImplementedError):
        fused["a"](xs["a"])  # nn.Module's own forward is back (FakeLinear defines none)


def test_fused_weight_requirements():
    mods = _modules()
    with pytest.raises(ValueError, match="one adapter_scale"):
        BatchedAdapters(mods, batch_factory=OracleBatch, out_dtype=torch.float32, fused_weight=True)
    mods = {"a": FakeLinear(40, 70, 6, 1)}
    with pytest.raises(ValueError, match="frozen base weights"):
        BatchedAdapters(mods, batch_factory=OracleBatch, out_dtype=torch.bfloat16, fused_weight=True)
    mods["a"].weight.requires_grad_(True)
    with pytest.raises(ValueError, match="frozen base weights"):
        BatchedAdapters(mods, batch_factory=OracleBatch, out_dtype=torch.float32, fused_weight=True)


def test_checkpoint_renders_without_model(tmp_path):
    mods = {"a": FakeLinear(40, 70, 6, 1, scale=0.5), "b": FakeLinear(64, 32, 9, 2, scale=0.5)}
    payload = {"format": "gaussian-peft-adapter", "step": 7,
               "metadata": {"adapter_config": {"adapter_scale": 0.5, "tile_out": 32, "tile_in": 32,
                                               "sigma_multiplier": 3.0, "normalize_gaussian": False,
                                               "init_method": "grid_overlap"}},
               "adapters": adapter_state_dict(mods)}
    path = tmp_path / "adapter.pt"
    torch.save(payload, path)
    loaded = torch.load(path, weights_only=False)
    cf = CheckpointFields(loaded, device="cpu", out_dtype=torch.float32, batch_factory=OracleBatch)
    assert cf.shapes == [(40, 70, 6), (64, 32, 9)] and cf.batch.out_scale == 0.5
    want = {n: d.detach().clone() for n, d in
            zip(mods, BatchedAdapters(mods, batch_factory=OracleBatch, out_dtype=torch.float32).render())}
    got = {n: d.clone() for n, d in cf.render().items()}
    for n in mods:
        assert torch.equal(got[n], want[n])
    # the adapters mapping alone works too (defaults: scale 1)
    cf1 = CheckpointFields(loaded["adapters"], device="cpu", out_dtype=torch.float32, batch_factory=OracleBatch)
    torch.testing.assert_close(cf1.render()["a"] * 0.5, want["a"], rtol=0, atol=0)
    # fused base weights
    w0 = {n: m.weight for n, m in mods.items()}
    cff = CheckpointFields(loaded, device="cpu", out_dtype=torch.float32, batch_factory=OracleBatch, base_weights=w0)
    for n, w in cff.render().items():
        torch.testing.assert_close(w, mods[n].weight + want[n], rtol=0, atol=1e-6)


def test_checkpoint_entries_checked():
    mods = {"a": FakeLinear(40, 70, 6, 1)}
    state = adapter_state_dict(mods)
    bad = {"a": dict(state["a"], num_gaussians=7)}
    with pytest.raises(ValueError, match="does not hold 7"):
        CheckpointFields(bad, device="cpu", batch_factory=OracleBatch)
    with pytest.raises(KeyError, match="amp"):
        CheckpointFields({"a": {k: v for k, v in state["a"].items() if k != "amp"}}, device="cpu",
                         batch_factory=OracleBatch)
    with pytest.raises(TypeError, match="unknown render settings"):
        CheckpointFields(state, device="cpu", batch_factory=OracleBatch, tile=16)
    with pytest.raises(ValueError, match="no adapter entries"):
        CheckpointFields({"format": "gaussian-peft-adapter", "adapters": {}}, device="cpu")
    with pytest.raises(ValueError, match="base weight"):
        CheckpointFields(state, device="cpu", batch_factory=OracleBatch, out_dtype=torch.float32,
                         base_weights={"a": torch.zeros(3, 3)})


def test_pair_capacity_bound_or_measured(monkeypatch):
    import guass_b200.adapters as A

    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    # 40x70: 2x3 tiles, 64x32: 2x1, 33x40: 2x2 (32x32 tiles)
    assert bank.batch.ids_capacity == 6 * 6 + 9 * 2 + 4 * 4
    bank.render()
    assert bank.batch.capacity_checks == 0
    monkeypatch.setattr(A, "MAX_BOUND_PAIRS", 10)
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    assert bank.batch.ids_capacity is None
    bank.render()
    bank.render()
    assert bank.batch.capacity_checks == 1  # measured once, on the first render


def test_render_publishes_layer_metadata():
    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    deltas = bank.render()
    for m, d in zip(mods.values(), deltas):
        md = m.last_forward_metadata
        assert md["execution_mode"] == "cuda_field_train" and md["accumulate_backend"] == "gfield_batched"
        # the norm of the unscaled delta, like GaussianLinear.compute_delta_weight
        want = float((d / m.adapter_config.adapter_scale).detach().float().norm())
        assert abs(md["delta_w_norm"] - want) <= 1e-5 * want
    quiet = _modules()
    BatchedAdapters(quiet, batch_factory=OracleBatch, track_metadata=False).render()
    assert not hasattr(quiet["a"], "last_forward_metadata")


def test_each_render_returns_its_own_delta():
    """A later render (here after a parameter change) must not overwrite the
    delta an earlier render returned: a graph that saved it keeps its values."""
    mods = _modules()
    bank = BatchedAdapters(mods, batch_factory=OracleBatch)
    first = bank.render()
    kept = [d.detach().clone() for d in first]
    with torch.no_grad():
        for m in mods.values():
            m.amp.mul_(3.0)
    second = bank.render()
    for a, b, c in zip(first, kept, second):
        assert torch.equal(a.detach(), b)
        assert not torch.equal(c.detach(), b)


def test_layer_metadata_resolves_norm_on_read():
    """The deferred delta_w_norm reads like the layer's plain dict: get(),
    dict() copies, ** unpacking and item access all see a float."""
    from guass_b200.adapters import _LayerMetadata, _PendingNorms

    norms = _PendingNorms(torch.tensor([1.5, 2.5]))
    base = {"execution_mode": "cuda_field_train"}
    for f, want in ((0, 1.5), (1, 2.5)):
        for read in (lambda m: m.get("delta_w_norm"), lambda m: dict(m)["delta_w_norm"],
                     lambda m: {**m}["delta_w_norm"], lambda m: m["delta_w_norm"],
                     lambda m: dict(m.items())["delta_w_norm"]):
            md = _LayerMetadata(base, norms, f)
            v = read(md)
            assert isinstance(v, float) and v == want
        md = _LayerMetadata(base, norms, f)
        assert len(md) == 2 and "delta_w_norm" in md and md == {**base, "delta_w_norm": want}
