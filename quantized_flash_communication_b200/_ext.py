"""Loader for the native extension ``_C`` (built in-tree by ``setup.py build_ext --inplace``).

CUDA tensors always go through the extension: if it is missing, the first CUDA call
raises instead of falling back to a slower path.  CPU tensors use the C++ CPU oracle
(also in ``_C``) or, without the extension, the torch specification in
``quantization.py``.

``count_launches()`` counts the kernels this package launches (for benchmark reports).
"""
from __future__ import annotations

import contextlib
import importlib

_C = None
_ERR: Exception | None = None
_COUNTING = None  # dict name -> calls while counting

# Kernels launched per call of an extension function (default 1).
# Host-only entries count 0; the fused GEMM + all-reduce entries launch the GEMM and the
# reduce kernel; decode attention launches its partial and merge kernels.
_KERNELS_PER_CALL = {"attn_decode": 2, "quantize_cpu": 0, "dequantize_cpu": 0, "pack_int4_cpu": 0,
                     "unpack_int4_cpu": 0, "ar_plan": 0, "ar_plan_rows": 0, "gemm_status": 0, "attn_status": 0,
                     "Workspace": 0, "set_nvtx": 0, "nvtx_enabled": 0, "set_norm_warps_per_row": 0, "set_attn_packed": 0, "set_two_shot_stages": 0, "set_gemv": 0, "gemm_all_reduce": 2, "gemm_all_reduce_norm": 2}


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


class _Counting:
    def __init__(self, mod, counts):
        self._mod = mod
        self._counts = counts

    def __getattr__(self, name):
        f = getattr(self._mod, name)
        if not callable(f) or name in ("Workspace",):
            return f
        counts = self._counts

        def wrapped(*a, **k):
            counts[name] = counts.get(name, 0) + 1
            return f(*a, **k)
        return wrapped


def ext():
    """The extension module; raises with build instructions if it failed to load."""
    m = _load()
    if m is None:
        raise RuntimeError(
            "quantized_flash_communication_b200._C is not built or failed to load "
            f"({_ERR!r}); run `python setup.py build_ext --inplace` at the repository root")
    if _COUNTING is not None:
        return _Counting(m, _COUNTING)
    return m


def has_ext() -> bool:
    return _load() is not None


@contextlib.contextmanager
def count_launches():
    """Within the block, count calls into the extension; yields a dict that receives
    ``{"calls": {name: n}, "kernels": total kernel launches}`` on exit."""
    global _COUNTING
    prev = _COUNTING
    _COUNTING = {}
    result = {}
    try:
        yield result
    finally:
        calls = dict(_COUNTING)
        _COUNTING = prev
        result["calls"] = calls
        result["kernels"] = sum(n * _KERNELS_PER_CALL.get(k, 1) for k, n in calls.items())
