"""SD1.5-shaped UNet training workload (guass_b200.sd15) on the CPU.

The adapters render through the oracle-backed batch double, so these tests
check the model layout, both ways of applying the delta, and the
data-parallel step (gloo ranks) -- not the CUDA kernels.
"""
from __future__ import annotations

import collections
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from guass_b200 import sd15, synthetic
from guass_b200.adapters import BatchedAdapters
from oracle_batch import OracleBatch


def test_full_layout_matches_the_render_workload():
    with torch.device("meta"):
        m = sd15.SD15UNet(sd15.UNetConfig())
    ad = m.adapters()
    assert len(ad) == 128
    got = collections.Counter((a.out_features, a.in_features) for a in ad.values())
    assert got == collections.Counter((o, i) for _, o, i in synthetic.unet_projection_shapes())
    assert all(a.mu_raw.shape == (256, 2) for a in ad.values())
    assert 855e6 < sum(p.numel() for p in m.parameters()) < 865e6  # SD1.5's UNet: ~860 M


def _model(seed=0):
    torch.manual_seed(seed)  # base weights of the non-adapter layers
    return sd15.SD15UNet(sd15.tiny_config(), dtype=torch.float32)


def _inputs(seed, batch=2):
    return sd15.synthetic_inputs(sd15.tiny_config(), batch, seed, dtype=torch.float32)


def _grads(model):
    return [p.grad.clone() for m in model.adapters().values() for p in (m.mu_raw, m.chol_raw, m.amp)]


def test_fused_and_reference_composition_agree():
    """One GEMM on W0 + delta vs the reference layer's base + row-chunked
    delta GEMMs: same loss and gradients up to fp32 rounding."""
    results = []
    for fused in (False, True):
        model = _model()
        bank = BatchedAdapters(model.adapters(), batch_factory=OracleBatch, out_dtype=torch.float32,
                               fused_weight=fused)
        bank.install()
        tr = sd15.DataParallelTrainer(model, bank)
        loss = tr.backward(_inputs(1))
        results.append((loss, _grads(model)))
    (l0, g0), (l1, g1) = results
    torch.testing.assert_close(l1, l0, rtol=1e-5, atol=0)
    for a, b in zip(g1, g0):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-6)


def test_unbound_projection_refuses():
    model = _model()
    x = torch.randn(1, 4, 32)
    blk = next(iter(model.adapters().values()))
    with pytest.raises(RuntimeError, match="BatchedAdapters"):
        blk(x[..., :blk.in_features])


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
        model = _model()
        bank = BatchedAdapters(model.adapters(), batch_factory=OracleBatch, out_dtype=torch.float32)
        bank.install()
        tr = sd15.DataParallelTrainer(model, bank, world=world)
        loss = tr.backward(_inputs(100 + rank))
        grads = _grads(model)
        tr.opt.step()
        params = [p.detach().clone() for p in tr.params]
        q.put((rank, float(loss), [g.numpy() for g in grads], [p.numpy() for p in params]))  # by value
    finally:
        dist.destroy_process_group()


def test_data_parallel_step_on_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (l, g, p)) for r, l, g, p in (q.get(timeout=300) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    # both ranks hold the averaged gradients and take the same optimizer step
    for a, b in zip(out[0][1], out[1][1]):
        assert (a == b).all()
    for a, b in zip(out[0][2], out[1][2]):
        assert (a == b).all()
    # averaged gradients == gradient of the mean of the two ranks' losses in one process
    model = _model()
    bank = BatchedAdapters(model.adapters(), batch_factory=OracleBatch, out_dtype=torch.float32)
    bank.install()
    tr = sd15.DataParallelTrainer(model, bank)
    bank.render()
    loss = sum(sd15.diffusion_loss(model, _inputs(100 + r), tr.alphas_cumprod) for r in range(2)) / 2
    loss.backward()
    torch.testing.assert_close(float(loss.detach()), (out[0][0] + out[1][0]) / 2, rtol=1e-6, atol=0)
    for a, b in zip(out[0][1], _grads(model)):
        torch.testing.assert_close(torch.from_numpy(a), b, rtol=1e-4, atol=1e-8)
