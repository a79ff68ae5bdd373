"""Loader for the native extension ``_C`` (built in-tree by ``setup.py build_ext --inplace``).

CUDA tensors always go through the extension: if it is missing, the first CUDA call
raises instead of falling back to a slower path.  CPU tensors use the C++ CPU oracle
(also in ``_C``) or, without the extension, the torch specification in
``quantization.py``.
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def _load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return _C
    try:
        import torch  # noqa: F401  (libtorch must be loaded before the extension)
        _C = importlib.import_module("quantized_flash_communication_b200._C")
    except Exception as e:  # pragma: no cover - exercised only when the build is missing
        _ERR = e
    return _C


def ext():
    """The extension module; raises with build instructions if it failed to load."""
    m = _load()
    if m is None:
        raise RuntimeError(
            "quantized_flash_communication_b200._C is not built or failed to load "
            f"({_ERR!r}); run `python setup.py build_ext --inplace` at the repository root")
    return m


def has_ext() -> bool:
    return _load() is not None
