"""Blockwise quantization: the pure-torch specification of every quantizer in this package.

This module is the numerical oracle. The CUDA kernels (``csrc/quant_kernels.cu``,
``csrc/allreduce.cu``, the GEMM epilogue) and the C++ CPU oracle (``csrc/quant_cpu.cpp``)
are tested bit-for-bit against the functions here.

Reference parity (file:line within the reference project):

* ``quantize_blockwise`` / ``dequantize_blockwise`` keep the names, arguments and
  return tuple of ``quantization.py:3-56``.
* The per-group arithmetic follows the Triton kernels of ``kernels.py:8-82``:
  asymmetric ``scale=(max-min)/qmax`` (``scale<1e-9`` -> 1), a clamped zero-point
  ``z=clamp(round(-min/scale),0,qmax)``, symmetric ``scale=absmax/(qmax/2)`` with a
  fixed offset ``(qmax+1)/2`` (``kernels.py:64-82`` does this for INT4 only; here INT8
  symmetric is defined the same way, 127.5 and 128).  Masked-off tail elements of a
  partial last group count as 0.0 in the min/max, as ``tl.load(..., other=0.0)`` does
  at ``kernels.py:13``.
* Rounding is half away from zero (libdevice ``round`` in the reference kernels),
  not torch's half-to-even.

Deliberate, documented differences from the reference:

* ``x/scale`` is computed as ``x * (1/scale)`` with an IEEE reciprocal, so that a GEMM
  epilogue can quantize 128 values with one divide.  A code can differ by one step
  from the reference's ``x/scale`` where ``x/scale`` lies within an ulp of a .5 boundary.
* The scale can be stored in fp16 (the reference's layout, ``kernels.py:30``) or fp32.
* Dequantized partial sums are accumulated in fp32 (the reference accumulates into an
  fp16 ``local_sum``, ``communication.py:52-59``).
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch

__all__ = [
    "rhaz",
    "qmax_for_bits",
    "phase_bits",
    "quantize_groups",
    "dequantize_groups",
    "pack_int4_ref",
    "unpack_int4_ref",
    "quantize_blockwise",
    "dequantize_blockwise",
    "two_step_all_reduce_ref",
    "one_shot_all_reduce_ref",
    "INT4_NIBBLE_ORDER",
]

# Nibble k (counting from the least significant bit) of a packed int32 word holds
# element INT4_NIBBLE_ORDER[k] of its 8-element block.  This is the reference's
# layout (kernels_jit.py:18-30): it lets the unpacker turn (word >> 4*i) & 0x000F000F
# into the half2 pair (e[2i], e[2i+1]) with one mask-or and one half2 subtract.
INT4_NIBBLE_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)

_SCALE_EPS = 1e-9


def qmax_for_bits(bits: int) -> int:
    if bits not in (4, 8):
        raise ValueError(f"quantized bit width must be 4 or 8, got {bits}")
    return (1 << bits) - 1


def phase_bits(bits: int) -> Tuple[int, int]:
    """Bit widths of the reduce-scatter and all-gather phases for a ``bits`` knob.

    16 -> no quantization, 8 -> INT8/INT8, 6 -> INT4 reduce-scatter + INT8 all-gather,
    4 -> INT4/INT4 (reference communication.py:30,64-67).
    """
    if bits == 16:
        return 16, 16
    if bits == 8:
        return 8, 8
    if bits == 6:
        return 4, 8
    if bits == 4:
        return 4, 4
    raise ValueError(f"bits must be one of 16, 8, 6, 4; got {bits}")


def rhaz(v: torch.Tensor) -> torch.Tensor:
    """Round half away from zero, exactly, in the tensor's own dtype."""
    t = torch.trunc(v)
    f = v - t  # exact in binary floating point
    return t + torch.where(f.abs() >= 0.5, torch.sign(v), torch.zeros_like(v))


def _grouped(x: torch.Tensor, group_size: int) -> Tuple[torch.Tensor, int]:
    flat = x.reshape(-1).to(torch.float32)
    n = flat.numel()
    pad = (-n) % group_size
    if pad:
        flat = torch.nn.functional.pad(flat, (0, pad))
    return flat.view(-1, group_size), pad


def quantize_groups(
    x: torch.Tensor,
    bits: int = 8,
    group_size: int = 128,
    mode: str = "asym",
    scale_dtype: torch.dtype = torch.float16,
):
    """Quantize ``x`` (any shape, any float dtype) group-wise along its flattened order.

    Returns ``(q, s, z)``: ``q`` uint8 codes ``[n]`` in ``0..2**bits-1`` (one code per
    byte, INT4 codes unpacked), ``s`` the per-group scale in ``scale_dtype`` and ``z``
    the per-group zero point as fp16 (an integer; ``(qmax+1)/2`` in symmetric mode).
    """
    qmax = float(qmax_for_bits(bits))
    g, pad = _grouped(x, group_size)
    if mode == "asym":
        mn = g.amin(dim=1, keepdim=True)
        mx = g.amax(dim=1, keepdim=True)
        s = (mx - mn) / qmax
        s = torch.where(s < _SCALE_EPS, torch.ones_like(s), s)
        inv = 1.0 / s
        z = torch.clamp(rhaz(-mn * inv), 0.0, qmax)
    elif mode == "sym":
        a = g.abs().amax(dim=1, keepdim=True)
        s = a / (qmax * 0.5)
        s = torch.where(s < _SCALE_EPS, torch.ones_like(s), s)
        inv = 1.0 / s
        z = torch.full_like(s, (qmax + 1.0) * 0.5)
    else:
        raise ValueError(f"mode must be 'asym' or 'sym', got {mode!r}")
    q = torch.clamp(rhaz(g * inv) + z, 0.0, qmax).to(torch.uint8).reshape(-1)
    n = q.numel() - pad
    return q[:n], s.reshape(-1).to(scale_dtype), z.reshape(-1).to(torch.float16)


def dequantize_groups(
    q: torch.Tensor,
    s: torch.Tensor,
    z: torch.Tensor,
    group_size: int = 128,
    out_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """``(q - z[g]) * s[g]`` in fp32, returned flat in ``out_dtype``."""
    if q.dtype == torch.int8:
        q = q.view(torch.uint8)
    qf = q.reshape(-1).to(torch.float32)
    n = qf.numel()
    pad = (-n) % group_size
    if pad:
        qf = torch.nn.functional.pad(qf, (0, pad))
    g = qf.view(-1, group_size)
    out = (g - z.to(torch.float32).view(-1, 1)) * s.to(torch.float32).view(-1, 1)
    return out.reshape(-1)[:n].to(out_dtype)


def pack_int4_ref(codes: torch.Tensor) -> torch.Tensor:
    """Pack 4-bit codes (one per byte) into int32 words, 8 codes per word.

    Pads with zeros to a multiple of 8 (reference kernels_jit.py:114-119).  Nibble k
    of a word holds element ``INT4_NIBBLE_ORDER[k]`` of its 8-element block.
    """
    c = codes.reshape(-1).to(torch.int64) & 0xF
    pad = (-c.numel()) % 8
    if pad:
        c = torch.nn.functional.pad(c, (0, pad))
    c = c.view(-1, 8)
    w = torch.zeros(c.shape[0], dtype=torch.int64, device=c.device)
    for k, e in enumerate(INT4_NIBBLE_ORDER):
        w |= c[:, e] << (4 * k)
    w = torch.where(w >= (1 << 31), w - (1 << 32), w)
    return w.to(torch.int32)


def unpack_int4_ref(words: torch.Tensor, numel: int | None = None) -> torch.Tensor:
    """Inverse of :func:`pack_int4_ref`; returns uint8 codes ``[numel]``."""
    w = words.reshape(-1).to(torch.int64) & 0xFFFFFFFF
    out = torch.empty(w.numel(), 8, dtype=torch.int64, device=w.device)
    for k, e in enumerate(INT4_NIBBLE_ORDER):
        out[:, e] = (w >> (4 * k)) & 0xF
    out = out.reshape(-1).to(torch.uint8)
    return out if numel is None else out[:numel]


# --------------------------------------------------------------------------------------
# Reference-compatible API (quantization.py:3-56)
# --------------------------------------------------------------------------------------
def quantize_blockwise(tensor: torch.Tensor, bits: int = 8, group_size: int = 128,
                       mode: str = "asym", scale_dtype: torch.dtype = torch.float32):
    """Same call and return tuple as the reference's ``quantize_blockwise``.

    Returns ``(quantized int8 [G, group_size], scale [G,1], zero_point [G,1],
    original_shape, pad_len)``; codes are stored as the uint8 bit pattern in int8.
    """
    original_shape = tensor.shape
    n = tensor.numel()
    pad_len = (-n) % group_size
    q, s, z = quantize_groups(tensor, bits, group_size, mode, scale_dtype)
    if pad_len:
        q = torch.nn.functional.pad(q, (0, pad_len))
    return (q.view(torch.int8).view(-1, group_size), s.view(-1, 1),
            z.to(torch.float32).view(-1, 1), original_shape, pad_len)


def dequantize_blockwise(quantized_data, scales, zero_points, original_shape, pad_len):
    """Same call as the reference's ``dequantize_blockwise``: ``(Q - Z) * S`` in fp32."""
    group_size = quantized_data.shape[-1]
    out = dequantize_groups(quantized_data.reshape(-1), scales.reshape(-1),
                            zero_points.reshape(-1), group_size, torch.float32)
    if pad_len:
        out = out[:-pad_len]
    return out.view(original_shape)


# --------------------------------------------------------------------------------------
# Whole-collective oracles, emulating W ranks in one process
# --------------------------------------------------------------------------------------
def _qdq(x: torch.Tensor, bits: int, group_size: int, mode: str, scale_dtype) -> torch.Tensor:
    if bits == 16:
        return x.reshape(-1).to(torch.float32)
    q, s, z = quantize_groups(x, bits, group_size, mode, scale_dtype)
    return dequantize_groups(q, s, z, group_size, torch.float32)


def two_step_all_reduce_ref(xs: Sequence[torch.Tensor], bits: int = 8, group_size: int = 128,
                            mode: str = "asym", scale_dtype=torch.float16,
                            out_dtype=None) -> torch.Tensor:
    """Two-step quantized all-reduce of ``xs[0..W-1]`` as every rank computes it.

    ``out = dq(q_p2( sum_j dq(q_p1(x_j)) ))`` with the sum in fp32 over ``j = 0..W-1``
    (reference communication.py:27-91).  Chunking never splits a group, so the
    chunk-local groups are the whole-tensor groups used here.
    """
    p1, p2 = phase_bits(bits)
    out_dtype = out_dtype or xs[0].dtype
    acc = None
    for x in xs:
        d = _qdq(x, p1, group_size, mode, scale_dtype)
        acc = d if acc is None else acc + d
    if p2 != 16:
        acc = _qdq(acc, p2, group_size, mode, scale_dtype)
    return acc.to(out_dtype).view(xs[0].shape)


def one_shot_all_reduce_ref(xs: Sequence[torch.Tensor], bits: int = 8, group_size: int = 128,
                            mode: str = "asym", scale_dtype=torch.float16,
                            out_dtype=None) -> torch.Tensor:
    """One-shot variant: every rank gathers all quantized inputs and sums them.

    ``out = sum_j dq(q(x_j))``: one quantization step, used for small messages.  For
    ``bits == 6`` the single step uses INT8 (the higher of the two widths).
    """
    p1, p2 = phase_bits(bits)
    b = max(p1, p2) if bits == 6 else p1
    out_dtype = out_dtype or xs[0].dtype
    acc = None
    for x in xs:
        d = _qdq(x, b, group_size, mode, scale_dtype)
        acc = d if acc is None else acc + d
    return acc.to(out_dtype).view(xs[0].shape)


def two_step_all_reduce_norm_ref(partials: Sequence[torch.Tensor], residual_shards: Sequence[torch.Tensor],
                                 weight: torch.Tensor, eps: float, bits: int = 8, group_size: int = 128,
                                 mode: str = "asym", scale_dtype=torch.float16):
    """Sequence-parallel all-reduce + residual + RMSNorm as the fused kernel computes it.

    Rank r owns rows ``[r*R, (r+1)*R)`` (``R = ceil(M/W)``) and holds them in
    ``residual_shards[r] [R, H]``.  ``sum = sum_j dq(q_p1(partial_j))`` (fp32, j in order);
    ``h = bf16(bf16(sum) + h)``; ``y = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w)``;
    every rank receives ``x = dq(q_p2(y))``.  Returns ``(x [M, H] bf16, new shards)``.
    """
    W = len(partials)
    M, H = partials[0].shape
    R = (M + W - 1) // W
    p1, p2 = phase_bits(bits)
    acc = None
    for x in partials:
        d = _qdq(x, p1, group_size, mode, scale_dtype).float()
        acc = d if acc is None else acc + d
    s_b = acc.view(M, H).to(torch.bfloat16).float()
    h = torch.cat([t.float() for t in residual_shards], 0)[:M]
    h = (s_b + h).to(torch.bfloat16).float()
    rstd = torch.rsqrt((h * h).sum(-1, keepdim=True) / H + eps)
    y = ((h * rstd).to(torch.bfloat16).float() * weight.float()).to(torch.bfloat16)
    x = _qdq(y, p2, group_size, mode, scale_dtype).view(M, H).to(torch.bfloat16) if p2 != 16 else y
    new = []
    for r in range(W):
        t = residual_shards[r].clone()
        n = max(0, min(M, (r + 1) * R) - r * R)
        t[:n] = h[r * R:r * R + n].to(t.dtype)
        new.append(t)
    return x.view(M, H), new


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().reshape(-1)
    b = b.double().reshape(-1)
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


__all__.append("rel_l2")

