"""Blockwise quantize / dequantize and INT4 pack / unpack operators.

CUDA tensors run the hand-written sm_100a kernels of ``csrc/quant_kernels.cu``; CPU
tensors run the C++ oracle of ``csrc/quant_cpu.cpp`` (or the torch specification in
``quantization.py`` when the extension is not built).  All three produce identical bits.
Reference capability: kernels.py:87-131 (quantize / dequantize) and kernels_jit.py:114-125
(pack / unpack).
"""
from __future__ import annotations

import torch

from .. import quantization as spec
from .._ext import ext, has_ext

__all__ = ["quantize", "dequantize", "pack_int4", "unpack_int4"]


def _check_mode(mode: str) -> bool:
    if mode not in ("asym", "sym"):
        raise ValueError(f"mode must be 'asym' or 'sym', got {mode!r}")
    return mode == "sym"


def quantize(x: torch.Tensor, bits: int = 8, group_size: int = 128, mode: str = "asym",
             scale_dtype: torch.dtype = torch.float16):
    """Quantize ``x`` in groups of ``group_size`` along its flattened order.

    Returns ``(q, s, z)``: uint8 codes ``[n]`` (one per byte; INT4 codes are 0..15),
    per-group scales ``[G]`` in ``scale_dtype`` (fp16 or fp32) and per-group zero points
    ``[G]`` in fp16.
    """
    sym = _check_mode(mode)
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    if scale_dtype not in (torch.float16, torch.float32):
        raise ValueError("scale_dtype must be torch.float16 or torch.float32")
    fp32 = scale_dtype == torch.float32
    if x.is_cuda:
        return tuple(ext().quantize(x, bits, group_size, sym, fp32))
    if has_ext():
        return tuple(ext().quantize_cpu(x, bits, group_size, sym, fp32))
    return spec.quantize_groups(x, bits, group_size, mode, scale_dtype)


def dequantize(q: torch.Tensor, s: torch.Tensor, z: torch.Tensor, group_size: int = 128,
               out_dtype: torch.dtype = torch.float16, shape=None) -> torch.Tensor:
    """``(q - z[g]) * s[g]``; ``q`` may hold uint8/int8 codes or fp16 codes."""
    if q.is_cuda:
        out = ext().dequantize(q.reshape(-1), s.reshape(-1), z.reshape(-1), group_size, out_dtype)
    elif has_ext():
        qq = q.reshape(-1)
        if qq.is_floating_point():
            qq = qq.to(torch.uint8)
        out = ext().dequantize_cpu(qq, s.reshape(-1), z.reshape(-1), group_size, out_dtype)
    else:
        qq = q.reshape(-1)
        if qq.is_floating_point():
            qq = qq.to(torch.uint8)
        out = spec.dequantize_groups(qq, s, z, group_size, out_dtype)
    return out if shape is None else out.view(shape)


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """8 one-byte 4-bit codes per int32 word (interleaved nibble order); zero-pads."""
    if codes.is_cuda:
        return ext().pack_int4(codes.reshape(-1))
    if has_ext():
        return ext().pack_int4_cpu(codes.reshape(-1))
    return spec.pack_int4_ref(codes)


def unpack_int4(words: torch.Tensor, numel: int) -> torch.Tensor:
    """int32 words -> ``numel`` fp16 codes (the reference's unpack output format)."""
    if words.is_cuda:
        return ext().unpack_int4(words.reshape(-1), int(numel))
    if has_ext():
        return ext().unpack_int4_cpu(words.reshape(-1), int(numel)).to(torch.float16)
    return spec.unpack_int4_ref(words, int(numel)).to(torch.float16)
