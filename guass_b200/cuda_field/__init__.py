"""Drop-in replacement for GUASS's ``gaussian_peft.cuda_field`` package.

Exports the same names as gaussian_peft/cuda_field/__init__.py.  To run an
existing GUASS model on this renderer without touching its layers, call
:func:`install` once after importing ``gaussian_peft``: it points the
reference runtime's ``load_extension`` at this package's extension object.
"""
from __future__ import annotations

from guass_b200.cuda_field.contracts import (
    NON_DIFFERENTIABLE_ARGS,
    SAVED_TENSOR_SPEC,
    STAGE0_THRESHOLDS,
    TENSOR_CONTRACT,
)
from guass_b200.cuda_field.loader import (
    CUDA_FIELD_EXTENSION_NAME,
    CUDA_FIELD_REFERENCE_EXTENSION_NAME,
    CUDA_FIELD_SOURCES,
    build_instructions,
    get_source_paths,
    load_extension,
)
from guass_b200.cuda_field.runtime import (
    gaussian_field_cuda_field_stage2_validation,
    gaussian_field_forward_reference,
    gaussian_field_reference,
    gaussian_field_train,
)


_ORIGINALS: dict = {}


def install(train_runtime: bool = True) -> None:
    """Route ``gaussian_peft.cuda_field`` (if importable) through this renderer.

    The reference runtime binds ``load_extension`` by name at import
    (gaussian_peft/cuda_field/runtime.py:8), so both the loader module and the
    runtime module are patched.  With ``train_runtime`` (default) the
    training entry point is also this package's ``gaussian_field_train``,
    which keeps the binning on the device (no pair-count read per layer);
    GaussianLinear binds that name at import (gaussian_linear.py:11), so the
    layer module's binding is replaced too.  :func:`uninstall` restores all."""
    import gaussian_peft.cuda_field.loader as ref_loader
    import gaussian_peft.cuda_field.runtime as ref_runtime

    targets = [(ref_loader, "load_extension", load_extension), (ref_runtime, "load_extension", load_extension)]
    if train_runtime:
        targets.append((ref_runtime, "gaussian_field_train", gaussian_field_train))
        try:
            import gaussian_peft.layers.gaussian_linear as ref_layer
            targets.append((ref_layer, "gaussian_field_train", gaussian_field_train))
        except ImportError:
            pass
    for mod, name, fn in targets:
        _ORIGINALS.setdefault((mod.__name__, name), (mod, getattr(mod, name)))
        setattr(mod, name, fn)


def uninstall() -> None:
    """Undo :func:`install`."""
    for (_, name), (mod, fn) in list(_ORIGINALS.items()):
        setattr(mod, name, fn)
    _ORIGINALS.clear()


__all__ = [
    "CUDA_FIELD_EXTENSION_NAME",
    "CUDA_FIELD_REFERENCE_EXTENSION_NAME",
    "CUDA_FIELD_SOURCES",
    "NON_DIFFERENTIABLE_ARGS",
    "SAVED_TENSOR_SPEC",
    "STAGE0_THRESHOLDS",
    "TENSOR_CONTRACT",
    "build_instructions",
    "gaussian_field_cuda_field_stage2_validation",
    "gaussian_field_forward_reference",
    "gaussian_field_reference",
    "gaussian_field_train",
    "get_source_paths",
    "install",
    "load_extension",
    "uninstall",
]
