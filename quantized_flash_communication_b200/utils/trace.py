"""Per-operator device timing for eager model steps, and NVTX ranges.

``OpTimer.region(name)`` brackets the kernels launched inside the ``with`` block by two
CUDA events on the current stream; ``summary()`` synchronizes once and returns, per
region name, the summed device milliseconds and the number of occurrences.  Meant for
eager runs (events inside a CUDA graph capture would be recorded into the graph); the
reference times its all-reduce with host ``perf_counter`` around two device syncs
(communication.py:8-96), which serializes the stream, whereas events do not.

NVTX: with ``QFC_NVTX=1`` in the environment (or ``set_nvtx(True)``) every model region
(``maybe_region``) and every CUDA op of the native extension pushes an NVTX range, so a
timeline tool shows each kernel under the layer step and the op that launched it.  The
ranges are host-side markers: they cost nothing on the device and are legal inside a
CUDA graph capture (they mark the capture, not the replays).
"""
from __future__ import annotations

import contextlib
import os
from collections import OrderedDict
from typing import Dict, List, Tuple

import torch


class OpTimer:
    def __init__(self):
        self._ev: "OrderedDict[str, List[Tuple[torch.cuda.Event, torch.cuda.Event]]]" = OrderedDict()

    @contextlib.contextmanager
    def region(self, name: str):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        try:
            yield
        finally:
            e.record()
            self._ev.setdefault(name, []).append((s, e))

    def reset(self):
        self._ev.clear()

    def names(self) -> List[str]:
        return list(self._ev.keys())

    def summary(self) -> Dict[str, Dict[str, float]]:
        torch.cuda.synchronize()
        out = OrderedDict()
        for name, pairs in self._ev.items():
            out[name] = {"ms": sum(s.elapsed_time(e) for s, e in pairs), "count": len(pairs)}
        return out


_nvtx_on = os.environ.get("QFC_NVTX", "0") == "1"


def set_nvtx(on: bool) -> None:
    """Turn NVTX ranges on or off, here and in the native extension's ops."""
    global _nvtx_on
    _nvtx_on = bool(on)
    from .._ext import _load
    m = _load()
    if m is not None:  # without the extension only the Python regions change
        m.set_nvtx(_nvtx_on)


def nvtx_enabled() -> bool:
    return _nvtx_on


@contextlib.contextmanager
def nvtx_range(name: str):
    """An NVTX range named ``name`` around the block (no-op while NVTX is off)."""
    if not _nvtx_on:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def _timed_nvtx(timer, name: str):
    with nvtx_range(name):
        if timer is None:
            yield
        else:
            with timer.region(name):
                yield


def maybe_region(timer, name: str):
    """``timer.region(name)`` when a timer is attached, plus an NVTX range while NVTX is
    on; a no-op context otherwise."""
    if timer is None and not _nvtx_on:
        return contextlib.nullcontext()
    return _timed_nvtx(timer, name)
