"""Device timing helpers: CUDA events on the launching stream, L2 flush between samples."""
from __future__ import annotations

from typing import Callable, List

import torch

_FLUSH = {}


def flush_l2(device=None):
    """Write a 256 MiB buffer (> the 126 MB L2 of a B200) so the next sample starts cold."""
    dev = torch.device(device or torch.cuda.current_device())
    buf = _FLUSH.get(dev)
    if buf is None:
        buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        _FLUSH[dev] = buf
    buf.fill_(1)


def time_fn(fn: Callable[[], object], iters: int = 20, warmup: int = 3, flush: bool = True) -> List[float]:
    """Per-iteration device times in ms (events bracket only ``fn``; the flush is outside)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return times


def median(xs):
    ys = sorted(xs)
    return ys[len(ys) // 2]
