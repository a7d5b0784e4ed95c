"""Loader of the compiled sm_100a kernel library (``vllm_sly_radiance_b200/_C*.so``).

CUDA tensors are only ever handed to these kernels: if the library is missing on a machine with
a GPU, every op raises instead of falling back to PyTorch."""
from __future__ import annotations

import importlib

import torch  # noqa: F401  (loads libc10 / libtorch, which the extension links against)

_EXT = None
_ERR = None


def ext():
    global _EXT, _ERR
    if _EXT is None:
        try:
            _EXT = importlib.import_module("vllm_sly_radiance_b200._C")
        except ImportError as e:   # pragma: no cover - depends on the build
            _ERR = e
            raise RuntimeError(
                "vllm_sly_radiance_b200._C is not built; run `python setup.py build_ext --inplace` "
                f"(import error: {e})") from e
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
