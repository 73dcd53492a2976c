"""Integration with GUASS's own package (CPU; skipped where it is absent).

The GPU box does not carry the reference, so these run in the build
container only: they check that `guass_b200.cuda_field.install()` routes the
reference runtime to this library, and that reference `GaussianLinear`
layers served by `BatchedAdapters` give the reference's own output.
"""
from __future__ import annotations

import sys

import pytest
import torch

from conftest import REFERENCE_ROOT as REF  # noqa: E402
if REF not in sys.path:
    sys.path.append(REF)
gp = pytest.importorskip("gaussian_peft")

from gaussian_peft.config.adapter import GaussianAdapterConfig  # noqa: E402
from gaussian_peft.layers.gaussian_linear import GaussianLinear  # noqa: E402

from oracle_batch import OracleBatch  # noqa: E402

from guass_b200 import cuda_field  # noqa: E402
from guass_b200.adapters import BatchedAdapters, adapter_state_dict  # noqa: E402


def test_install_routes_reference_runtime_to_this_library():
    import gaussian_peft.cuda_field.loader as ref_loader
    import gaussian_peft.cuda_field.runtime as ref_runtime

    import gaussian_peft.layers.gaussian_linear as ref_layer

    saved = (ref_loader.load_extension, ref_runtime.load_extension, ref_runtime.gaussian_field_train,
             ref_layer.gaussian_field_train)
    args = dict(row_coords=torch.linspace(-1, 1, 8), col_coords=torch.linspace(-1, 1, 9), mu=torch.zeros(2, 2),
                chol_raw=torch.zeros(2, 3), amp=torch.zeros(2, 1), tile_out=32, tile_in=32, sigma_multiplier=3.0)
    try:
        cuda_field.install(train_runtime=False)
        assert ref_runtime.load_extension is cuda_field.load_extension
        ext = ref_runtime.load_extension()
        assert type(ext).__module__ == "guass_b200.cuda_field._ext"
        assert ref_layer.gaussian_field_train is saved[3]
        # the reference's own train function now reaches our argument checks
        with pytest.raises(RuntimeError, match="row_coords must be a CUDA tensor"):
            ref_runtime.gaussian_field_train(**args)
        cuda_field.uninstall()
        cuda_field.install()  # default: the layers call this package's training function
        assert ref_layer.gaussian_field_train is cuda_field.gaussian_field_train
        assert ref_runtime.gaussian_field_train is cuda_field.gaussian_field_train
        with pytest.raises(RuntimeError, match="row_coords must be a CUDA tensor"):
            ref_layer.gaussian_field_train(**args)
        cuda_field.uninstall()
        assert (ref_loader.load_extension, ref_runtime.load_extension, ref_runtime.gaussian_field_train,
                ref_layer.gaussian_field_train) == saved
    finally:
        cuda_field.uninstall()
        (ref_loader.load_extension, ref_runtime.load_extension, ref_runtime.gaussian_field_train,
         ref_layer.gaussian_field_train) = saved


def _layer(out_f, in_f, k, seed):
    torch.manual_seed(seed)
    cfg = GaussianAdapterConfig(init_num_gaussians=k, init_method="random_uniform", init_amp_scale=1e-2,
                                execution_mode="tiled_reference_pytorch")
    layer = GaussianLinear(in_f, out_f, adapter_config=cfg)
    return layer


def test_batched_adapters_serve_reference_layers():
    layers = {"q": _layer(48, 64, 12, 0), "k": _layer(48, 40, 9, 1)}
    x = torch.randn(3, 64), torch.randn(3, 40)
    want = [layers["q"](x[0]), layers["k"](x[1])]  # reference path, per layer
    bank = BatchedAdapters(layers, batch_factory=OracleBatch, out_dtype=torch.float32)
    bank.install()
    try:
        bank.render()
        got = [layers["q"](x[0]), layers["k"](x[1])]
    finally:
        bank.uninstall()
    for a, b in zip(got, want):
        assert torch.allclose(a, b, rtol=1e-4, atol=1e-6)
    st = adapter_state_dict(layers)
    assert st["q"]["num_gaussians"] == 12 and st["k"]["in_features"] == 40


def test_merge_into_reference_weights():
    layers = {"q": _layer(48, 64, 12, 0)}
    x = torch.randn(3, 64)
    want = layers["q"](x)
    w0 = layers["q"].weight.detach().clone()
    bank = BatchedAdapters(layers, batch_factory=OracleBatch, out_dtype=torch.float32)
    bank.merge_into_weights()
    try:
        assert torch.allclose(layers["q"](x), want, rtol=1e-4, atol=1e-6)
        assert not torch.equal(layers["q"].weight, w0)
    finally:
        bank.unmerge_weights()
        bank.uninstall()
    assert torch.allclose(layers["q"].weight, w0, atol=1e-7)


def test_model_renderer_serves_a_reference_model():
    """One batched render per model forward for a model of reference
    GaussianLinear layers: same output and gradients as the layers' own path."""
    from guass_b200.adapters import ModelRenderer

    def model():
        torch.manual_seed(0)
        return torch.nn.Sequential(_layer(40, 64, 12, 0), torch.nn.GELU(), _layer(24, 40, 9, 1))

    x = torch.randn(5, 64)
    ref = model()
    want = ref(x)
    want.square().sum().backward()
    m = model()
    r = ModelRenderer(m, batch_factory=OracleBatch, out_dtype=torch.float32)
    try:
        got = m(x)
        got.square().sum().backward()
        assert r.bank.batch.calls == 1
        torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-6)
        for a, b in zip(m.parameters(), ref.parameters()):
            if b.grad is not None:
                torch.testing.assert_close(a.grad, b.grad, rtol=1e-3, atol=1e-6)
        m(x)
        assert r.bank.batch.calls == 2  # one render per model forward
    finally:
        r.remove()
    assert m[0].compute_delta_weight.__func__ is GaussianLinear.compute_delta_weight
