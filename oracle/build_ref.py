"""Build GUASS's own cuda_field extension from its sources into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The reference's CUDA path
(gaussian_peft/cuda_field/csrc/{ext.cpp, field_impl.cu, forward.cu,
backward.cu}) is compiled where it lies, unmodified, with the reference's own
-O2 (gaussian_peft/cuda_field/setup.py:48-51) plus an sm_100a target.  Nothing
is copied into this repository; the build products stay in oracle/_ref/,
which git ignores but which travels to the GPU box.

The GPU parity tests load the result with :func:`load` and compare the
product path against it on identical inputs.  The reference's own loader is
not used because it writes into the (read-only) reference tree
(gaussian_peft/cuda_field/loader.py:15-16,82-93).

Usage (in the build container, where the reference sources are mounted):
    python oracle/build_ref.py [--src /path/to/reference]
"""
from __future__ import annotations

import argparse
import glob
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
MODULE_NAME = "gaussian_peft_cuda_field_reference"  # loader.py:10-11
# GUASS project root (the reference sources); override with GUASS_REFERENCE_ROOT
DEFAULT_SRC = os.environ.get("GUASS_REFERENCE_ROOT", "/root/reference")


def build(src_root: str = DEFAULT_SRC, verbose: bool = False) -> Path | None:
    csrc = Path(src_root) / "gaussian_peft" / "cuda_field" / "csrc"
    if not csrc.is_dir():
        return None
    from torch.utils.cpp_extension import load

    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    build_dir = REF_OUT / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    load(
        name=MODULE_NAME,
        sources=[str(csrc / f) for f in ("ext.cpp", "field_impl.cu", "forward.cu", "backward.cu")],
        extra_cflags=["-O2"],
        extra_cuda_cflags=["-O2", "-gencode", "arch=compute_100a,code=sm_100a"],
        build_directory=str(build_dir),
        verbose=verbose,
    )
    return find_module()


def find_module() -> Path | None:
    hits = sorted(glob.glob(str(REF_OUT / "build" / f"{MODULE_NAME}*.so")))
    return Path(hits[-1]) if hits else None


def load():
    """Import the prebuilt reference extension (requires torch imported)."""
    import torch  # noqa: F401  (the extension links against libtorch)

    if MODULE_NAME in sys.modules:
        return sys.modules[MODULE_NAME]
    path = find_module()
    if path is None:
        raise FileNotFoundError("reference extension not built: run python oracle/build_ref.py")
    spec = importlib.util.spec_from_file_location(MODULE_NAME, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[MODULE_NAME] = mod
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=DEFAULT_SRC)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    out = build(a.src, a.verbose)
    print(out if out else "reference sources not found; nothing built")
