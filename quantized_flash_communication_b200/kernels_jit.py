"""Reference-compatible INT4 pack / unpack (reference kernels_jit.py:114-125).

Same layout bit for bit: 8 codes per int32 word, nibble k (from the LSB) holding
element ``[0,2,4,6,1,3,5,7][k]`` of its block; unpack returns the codes as fp16.  The
kernels are built ahead of time (``setup.py``) rather than at import, and launch on the
caller's current stream rather than the legacy default stream.
"""
from __future__ import annotations

import torch

from .ops import quant as _q

__all__ = ["pack_int4", "unpack_int4"]


def pack_int4(q_tensor: torch.Tensor) -> torch.Tensor:
    """One-byte 4-bit codes -> int32 words ``[ceil(n/8)]`` (zero-padded)."""
    return _q.pack_int4(q_tensor)


def unpack_int4(packed_tensor: torch.Tensor, original_shape) -> torch.Tensor:
    """int32 words -> fp16 codes of ``original_shape``."""
    shape = torch.Size(original_shape)
    return _q.unpack_int4(packed_tensor, shape.numel()).view(shape)
