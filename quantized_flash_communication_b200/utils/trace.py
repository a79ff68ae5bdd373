"""Per-operator device timing for eager model steps.

``OpTimer.region(name)`` brackets the kernels launched inside the ``with`` block by two
CUDA events on the current stream; ``summary()`` synchronizes once and returns, per
region name, the summed device milliseconds and the number of occurrences.  Meant for
eager runs (events inside a CUDA graph capture would be recorded into the graph); the
reference times its all-reduce with host ``perf_counter`` around two device syncs
(communication.py:8-96), which serializes the stream, whereas events do not.
"""
from __future__ import annotations

import contextlib
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


def maybe_region(timer, name: str):
    """``timer.region(name)`` when a timer is attached, else a no-op context."""
    return timer.region(name) if timer is not None else contextlib.nullcontext()
