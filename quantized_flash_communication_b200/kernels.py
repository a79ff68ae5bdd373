"""Reference-compatible quantizer entry points (reference kernels.py:87-131).

``triton_quantize`` / ``triton_dequantize`` keep the reference's names, arguments and
outputs (int8 codes one per byte, fp16 scale and zero point per group), but run the
hand-written sm_100a CUDA kernels of ``csrc/quant_kernels.cu`` (no Triton).  Symmetric
INT8 is a real mode here (absmax / 127.5, offset 128); the reference's dispatcher
launches nothing for it (kernels.py:97-104).
"""
from __future__ import annotations

import torch

from .ops import quant as _q

__all__ = ["triton_quantize", "triton_dequantize", "quantize", "dequantize"]

quantize = _q.quantize
dequantize = _q.dequantize


def triton_quantize(x: torch.Tensor, bits: int = 8, block_size: int = 128, mode: str = "asym"):
    """Returns ``(q int8 [n], s fp16 [G], z fp16 [G])`` like the reference.

    ``bits <= 4`` selects the 4-bit quantizer (codes stay one per byte), as in the
    reference (kernels.py:99-102).
    """
    b = 8 if bits == 8 else 4
    if bits not in (8,) and bits > 4:
        raise ValueError(f"bits must be 8 or <= 4, got {bits}")
    q, s, z = _q.quantize(x, b, block_size, mode, torch.float16)
    return q.view(torch.int8), s, z


def triton_dequantize(q_x: torch.Tensor, s_x: torch.Tensor, z_x: torch.Tensor, original_shape,
                      block_size: int = 128) -> torch.Tensor:
    """``(q - z) * s`` as fp16 in ``original_shape``; ``q`` may be int8 or fp16 codes."""
    n = q_x.numel()
    out = _q.dequantize(q_x, s_x, z_x, block_size, torch.float16)
    return out[:n].view(original_shape)
