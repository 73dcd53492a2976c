"""Extension loader with the reference loader's public names.

Mirrors gaussian_peft/cuda_field/loader.py:96-109: ``load_extension()`` returns
the (cached) extension object whose three methods the runtime calls.  The
object is backed by the in-tree libgfield.so; a missing library raises
ImportError instead of building or falling back.
"""
from __future__ import annotations

from functools import lru_cache
from pathlib import Path

from guass_b200 import _lib

CUDA_FIELD_EXTENSION_NAME = "guass_b200_gfield"
CUDA_FIELD_REFERENCE_EXTENSION_NAME = CUDA_FIELD_EXTENSION_NAME
CUDA_FIELD_SOURCES = (Path(__file__).resolve().parent.parent / "csrc" / "gfield.cu",)


def get_source_paths() -> list[str]:
    return [str(p) for p in CUDA_FIELD_SOURCES]


def build_instructions() -> str:
    return ("B200 Gaussian-field renderer: build libgfield.so with `python -m guass_b200._build` "
            f"(nvcc, sm_100a). Sources: {', '.join(get_source_paths())}; library: {_lib.LIB_PATH}")


def load_extension(*, verbose: bool = False):
    """The one extension object of this process (``verbose`` is accepted for
    the reference's signature; nothing is built here)."""
    return _extension()


@lru_cache(maxsize=1)
def _extension():
    from guass_b200.cuda_field._ext import GaussianFieldExtension

    return GaussianFieldExtension()
