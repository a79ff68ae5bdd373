"""Reference-compatible communication entry point (reference communication.py:7-97).

``flash_all_reduce(tensor, group_size=128, bits=8, quant_type="asym") -> (tensor, ms)``
keeps the reference's call, knobs and return tuple:

* ``bits``: 16 = unquantized, 8 = INT8/INT8, 6 = INT4 reduce-scatter + INT8 all-gather,
  4 = INT4/INT4;
* ``quant_type``: "asym" (min/max) or "sym" (absmax, fixed offset);
* the result is fp16 for quantized calls and the input itself (all-reduced in place) for
  ``bits == 16``; ``ms`` is the host-timed latency between two device synchronisations.

Underneath, a CUDA tensor goes through ONE fused sm_100a kernel that moves quantized
chunks over NVLink with peer stores (``parallel/quant_allreduce.py``); there is no NCCL
call on the data path.  CPU tensors (gloo) and group sizes above 256 take the staged
path of ``parallel/staged.py``.  Extra keyword-only knobs: ``group`` (process group),
``out_dtype``, ``inplace``, ``algo`` ("two_shot" = the reference's semantics, "one_shot",
"auto"), ``timing`` ("host" = the reference's synchronised timing, "none" = no sync,
``ms`` = 0), ``scale_dtype`` (fp16 as in the reference, or fp32) and ``backend``
("auto", "fused", "staged", "nccl" = plain NCCL all-reduce for ``bits == 16``).
"""
from __future__ import annotations

import time
from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from .parallel.quant_allreduce import QuantAllReduce
from .parallel.staged import staged_all_reduce

__all__ = ["flash_all_reduce", "get_quant_all_reduce", "reset_communicators"]

_CACHE: Dict[tuple, QuantAllReduce] = {}


def get_quant_all_reduce(group: Optional[dist.ProcessGroup] = None, device=None,
                         scale_dtype: torch.dtype = torch.float16) -> QuantAllReduce:
    """The cached fused all-reduce (and its peer-mapped workspace) of a process group."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    key = (id(group), device.index, scale_dtype)
    ar = _CACHE.get(key)
    if ar is None:
        ar = QuantAllReduce(group, device, scale_dtype=scale_dtype, algo="two_shot")
        _CACHE[key] = ar
    return ar


def reset_communicators():
    """Drop cached workspaces (call before destroying their process groups)."""
    torch.cuda.synchronize() if torch.cuda.is_available() else None
    _CACHE.clear()


def flash_all_reduce(tensor: torch.Tensor, group_size: int = 128, bits: int = 8, quant_type: str = "asym", *,
                     group: Optional[dist.ProcessGroup] = None, out_dtype: Optional[torch.dtype] = torch.float16,
                     inplace: bool = False, algo: str = "two_shot", timing: str = "host",
                     scale_dtype: torch.dtype = torch.float16, backend: str = "auto") -> Tuple[torch.Tensor, float]:
    if timing not in ("host", "none"):
        raise ValueError("timing must be 'host' or 'none'")
    if timing == "host" and tensor.is_cuda:
        torch.cuda.synchronize()
    t0 = time.perf_counter()

    if bits == 16 or inplace or out_dtype is None:
        od = tensor.dtype
    else:
        od = out_dtype
    if bits == 16 and backend == "nccl":
        dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=group)
        out = tensor
    elif tensor.is_cuda and backend in ("auto", "fused") and 8 <= group_size <= 256:
        ar = get_quant_all_reduce(group, tensor.device, scale_dtype)
        dst = tensor if (bits == 16 or inplace) and tensor.is_contiguous() and od == tensor.dtype else None
        out = ar(tensor, out=dst, out_dtype=od, bits=bits, group_size=group_size, quant_type=quant_type,
                 algo=algo)
    elif backend in ("auto", "staged"):
        out = staged_all_reduce(tensor, bits, group_size, quant_type, scale_dtype, group, od)
        if bits == 16 or inplace:
            tensor.copy_(out.view(tensor.shape))
            out = tensor
    else:
        raise ValueError(f"backend {backend!r} cannot run this call (bits={bits}, group_size={group_size}, "
                         f"device={tensor.device})")

    if timing == "host":
        if tensor.is_cuda:
            torch.cuda.synchronize()
        ms = (time.perf_counter() - t0) * 1000.0
    else:
        ms = 0.0
    return out.view(tensor.shape), ms
