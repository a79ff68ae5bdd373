"""Two-step quantized all-reduce built from torch.distributed collectives.

The same algorithm as the fused kernel (and bit-identical to it and to the oracle in
``quantization.py``), expressed with ``all_to_all_single`` (the reduce-scatter of
quantized chunks) and ``all_gather_into_tensor``.  It serves

* CPU / gloo process groups (plumbing without a GPU; gloo lacks the list ``all_to_all``
  the reference uses at communication.py:48-50, but has ``all_to_all_single``);
* group sizes above 256, which the fused kernel does not take (the reference's
  perplexity sweep goes to 8192, main.py:87);
* an NCCL baseline with the reference's structure for comparisons.

Unlike the reference, payload, scales and zero points of a chunk travel in one byte
buffer, so each phase is a single collective instead of three.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import quantization as spec
from ..ops import quant as Q

__all__ = ["staged_all_reduce"]


def _encode(x: torch.Tensor, bits: int, gs: int, mode: str, scale_dtype, n_chunks: int) -> torch.Tensor:
    """Quantize a flat tensor (length multiple of gs * n_chunks) into [n_chunks, bytes]."""
    if bits == 16:
        return x.reshape(n_chunks, -1).contiguous().view(torch.uint8).reshape(n_chunks, -1)
    q, s, z = Q.quantize(x, bits, gs, mode, scale_dtype)
    if bits == 4:
        q = Q.pack_int4(q).view(torch.uint8)
    q = q.reshape(n_chunks, -1)
    s = s.contiguous().view(torch.uint8).reshape(n_chunks, -1)
    z = z.contiguous().view(torch.uint8).reshape(n_chunks, -1)
    return torch.cat([q, s, z], dim=1).contiguous()


def _decode(buf: torch.Tensor, bits: int, gs: int, chunk: int, wire_dtype, scale_dtype) -> torch.Tensor:
    """[k, bytes] -> fp32 values [k, chunk]."""
    k = buf.shape[0]
    if bits == 16:
        return buf.contiguous().view(wire_dtype).reshape(k, chunk).to(torch.float32)
    pay = chunk if bits == 8 else chunk // 2
    G = chunk // gs
    sb = G * (4 if scale_dtype == torch.float32 else 2)
    out = torch.empty(k, chunk, dtype=torch.float32, device=buf.device)
    for i in range(k):
        row = buf[i]
        q = row[:pay].contiguous()
        s = row[pay:pay + sb].contiguous().view(scale_dtype)
        z = row[pay + sb:pay + sb + 2 * G].contiguous().view(torch.float16)
        if bits == 4:
            q = Q.unpack_int4(q.view(torch.int32), chunk)
        out[i] = Q.dequantize(q, s, z, gs, torch.float32)
    return out


def staged_all_reduce(x: torch.Tensor, bits: int = 8, group_size: int = 128, mode: str = "asym",
                      scale_dtype: torch.dtype = torch.float16, group: Optional[dist.ProcessGroup] = None,
                      out_dtype: Optional[torch.dtype] = None, quantize_local: bool = True) -> torch.Tensor:
    """Two-step quantized all-reduce of ``x`` over ``group``; returns a new tensor."""
    W = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    out_dtype = out_dtype or x.dtype
    p1, p2 = spec.phase_bits(bits)
    flat = x.reshape(-1)
    n = flat.numel()
    align = group_size * W * 8  # chunks of whole groups and whole INT4 words
    pad = (-n) % align
    if pad:
        flat = torch.nn.functional.pad(flat, (0, pad))
    chunk = flat.numel() // W
    wire = x.dtype

    # Phase 1: reduce-scatter of quantized chunks (one all-to-all).
    send = _encode(flat, p1, group_size, mode, scale_dtype, W)
    if W > 1:
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
    else:
        recv = send
    vals = _decode(recv, p1, group_size, chunk, wire, scale_dtype)
    if not quantize_local:
        vals[rank] = flat[rank * chunk:(rank + 1) * chunk].to(torch.float32)
    acc = vals[0].clone()
    for j in range(1, W):
        acc = acc + vals[j]

    # Phase 2: all-gather of the requantized reduced chunk (one all-gather).
    if p2 == 16:
        acc = acc.to(wire)
    mine = _encode(acc, p2, group_size, mode, scale_dtype, 1)
    if W > 1:
        gathered = torch.empty(W * mine.numel(), dtype=torch.uint8, device=mine.device)
        dist.all_gather_into_tensor(gathered, mine.reshape(-1), group=group)
        gathered = gathered.view(W, -1)
    else:
        gathered = mine
    out = _decode(gathered, p2, group_size, chunk, wire, scale_dtype).reshape(-1)[:n]
    return out.to(out_dtype).view(x.shape)
