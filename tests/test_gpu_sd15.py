"""The SD1.5 adapter training workload (guass_b200.sd15) on the CUDA batch,
at the tiny layout: both ways of applying the delta agree, a bf16 step runs,
and the adapter gradients reach every Gaussian parameter."""
from __future__ import annotations

import pytest
import torch

from guass_b200 import sd15
from guass_b200.adapters import BatchedAdapters

pytestmark = pytest.mark.gpu


def _setup(fused, dtype):
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = sd15.SD15UNet(sd15.tiny_config(), dtype=dtype)
    model.cuda()
    bank = BatchedAdapters(model.adapters(), out_dtype=dtype, fused_weight=fused)
    bank.install()
    return model, bank, sd15.DataParallelTrainer(model, bank)


def _grads(model):
    return [p.grad.clone() for m in model.adapters().values() for p in (m.mu_raw, m.chol_raw, m.amp)]


def test_fused_and_reference_composition_agree_fp32(monkeypatch):
    # plain fp32 everywhere (cuDNN would otherwise run the convolutions in TF32)
    monkeypatch.setattr(torch.backends.cudnn, "allow_tf32", False)
    monkeypatch.setattr(torch.backends.cuda.matmul, "allow_tf32", False)
    out = []
    for fused in (False, True):
        model, bank, tr = _setup(fused, torch.float32)
        loss = tr.backward(sd15.synthetic_inputs(sd15.tiny_config(), 2, 1, device="cuda", dtype=torch.float32))
        assert bank.batch.device_flags() == 0
        out.append((loss, _grads(model)))
    torch.testing.assert_close(out[1][0], out[0][0], rtol=1e-4, atol=0)
    for a, b in zip(out[1][1], out[0][1]):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-5)


@pytest.mark.parametrize("fused", [False, True])
def test_bf16_training_steps(fused):
    model, bank, tr = _setup(fused, torch.bfloat16)
    inp = sd15.synthetic_inputs(sd15.tiny_config(), 2, 2, device="cuda")
    for _ in range(3):
        loss = tr.step(inp)
    torch.cuda.synchronize()
    assert torch.isfinite(loss).item()
    assert bank.batch.device_flags() == 0
    tr.backward(inp)
    # every adapter's mu_raw, chol_raw and amp receives a non-zero, finite gradient
    for p in tr.params:
        assert torch.isfinite(p.grad).all() and p.grad.abs().sum() > 0


def test_per_layer_dropin_matches_batched_render_fp32(monkeypatch):
    """Every layer rendering itself through the drop-in runtime (the
    reference's call pattern) gives the loss and gradients of the batched
    render with the same layer composition."""
    monkeypatch.setattr(torch.backends.cudnn, "allow_tf32", False)
    monkeypatch.setattr(torch.backends.cuda.matmul, "allow_tf32", False)
    out = []
    for mode in ("batched", "dropin"):
        torch.manual_seed(0)
        with torch.device("cuda"):
            model = sd15.SD15UNet(sd15.tiny_config(), dtype=torch.float32)
        model.cuda()
        if mode == "dropin":
            bank = sd15.PerLayerRender(model.adapters())
        else:
            bank = BatchedAdapters(model.adapters(), out_dtype=torch.float32)
        bank.install()
        tr = sd15.DataParallelTrainer(model, bank)
        loss = tr.backward(sd15.synthetic_inputs(sd15.tiny_config(), 2, 3, device="cuda", dtype=torch.float32))
        out.append((loss, _grads(model)))
    torch.testing.assert_close(out[1][0], out[0][0], rtol=1e-5, atol=0)
    for a, b in zip(out[1][1], out[0][1]):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-7)


def test_model_renderer_matches_per_layer_render_fp32(monkeypatch):
    """ModelRenderer (one batched render per model forward, from a pre-hook)
    gives the per-layer drop-in path's loss and gradients."""
    from guass_b200.adapters import ModelRenderer

    monkeypatch.setattr(torch.backends.cudnn, "allow_tf32", False)
    monkeypatch.setattr(torch.backends.cuda.matmul, "allow_tf32", False)
    inp = sd15.synthetic_inputs(sd15.tiny_config(), 2, 4, device="cuda", dtype=torch.float32)
    out = []
    for mode in ("dropin", "hook"):
        torch.manual_seed(0)
        with torch.device("cuda"):
            model = sd15.SD15UNet(sd15.tiny_config(), dtype=torch.float32)
        model.cuda()
        if mode == "dropin":
            sd15.PerLayerRender(model.adapters()).install()
        else:
            renderer = ModelRenderer(model, out_dtype=torch.float32)
        loss = sd15.diffusion_loss(model, inp, sd15.noise_schedule("cuda"))
        loss.backward()
        out.append((loss.detach(), _grads(model)))
    renderer.remove()
    torch.testing.assert_close(out[1][0], out[0][0], rtol=1e-5, atol=0)
    for a, b in zip(out[1][1], out[0][1]):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-7)
