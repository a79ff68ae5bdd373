"""Llama layer operators on the sm_100a kernels of ``csrc/layers.cu``."""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import ext

__all__ = ["rmsnorm", "rope_kv", "silu_mul", "embedding", "argmax", "rope_cos_sin"]


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``rmsnorm(x [+ residual]) * w``; with ``residual``, it is updated in place to x + residual."""
    y = torch.empty_like(x) if out is None else out
    ext().rmsnorm(x, residual, w, y, eps)
    return y


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, device, scaling: Optional[dict] = None) -> torch.Tensor:
    """fp32 table [max_pos, head_dim/2, 2] of (cos, sin) for the rotate-half convention."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling is not None and scaling.get("rope_type") == "llama3":
        # Llama-3.1 frequency scaling (long-context wavelength bands).
        factor = scaling["factor"]
        lo, hi = scaling["low_freq_factor"], scaling["high_freq_factor"]
        old = scaling["original_max_position_embeddings"]
        wavelen = 2 * torch.pi / inv
        smooth = (old / wavelen - lo) / (hi - lo)
        scaled = torch.where(wavelen > old / lo, inv / factor, inv)
        mid = (wavelen <= old / lo) & (wavelen >= old / hi)
        inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.stack([f.cos(), f.sin()], dim=-1).to(torch.float32).to(device).contiguous()


def rope_kv(qkv: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor, nq: int, nkv: int, hd: int,
            k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None,
            slot_mapping: Optional[torch.Tensor] = None) -> None:
    """In-place RoPE on q and k of ``qkv [M, (nq+2nkv)*hd]``; optionally writes k, v to the paged cache."""
    ext().rope_kv(qkv, pos, cos_sin, k_cache, v_cache, slot_mapping, nq, nkv, hd)


def rope_kv_decode(qkv: torch.Tensor, cos_sin: torch.Tensor, nq: int, nkv: int, hd: int, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor) -> None:
    """In-place RoPE of one decode token per sequence (``qkv [B, (nq+2nkv)*hd]``) at position
    ``seq_lens[b] - 1``, and its k, v written to the paged cache through ``block_table``;
    positions and cache slots are computed inside the kernel."""
    ext().rope_kv_decode(qkv, cos_sin, k_cache, v_cache, block_table, seq_lens, nq, nkv, hd)


def silu_mul(gu: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    I = gu.shape[-1] // 2
    y = torch.empty(*gu.shape[:-1], I, dtype=gu.dtype, device=gu.device) if out is None else out
    ext().silu_mul(gu, y)
    return y


def embedding(ids: torch.Tensor, table: torch.Tensor, vocab_start: int = 0,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rows of ``table`` for ``ids`` (rows outside [vocab_start, vocab_start+V) read as zero)."""
    y = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device) if out is None else out
    ext().embedding(ids.reshape(-1), table, y, vocab_start)
    return y


def argmax(logits: torch.Tensor, idx_offset: int = 0, valid: Optional[int] = None,
           rng: Optional[torch.Tensor] = None, inv_temp: float = 1.0, done: Optional[torch.Tensor] = None):
    """Row-wise (max score fp32, argmax int64 + idx_offset) of ``logits [M, V]``.

    Only the first ``valid`` columns take part (all by default).  With ``rng`` (int64
    [seed, step] on the device) the score is ``logit * inv_temp`` plus Gumbel noise, so the
    argmax is a sample from softmax(logit * inv_temp); the kernel then advances the step
    (``done``: an int32 arrival counter on the device, zero before the first call).
    """
    M = logits.shape[0]
    bv = torch.empty(M, dtype=torch.float32, device=logits.device)
    bi = torch.empty(M, dtype=torch.int64, device=logits.device)
    ext().argmax(logits, bv, bi, idx_offset, -1 if valid is None else int(valid), rng, float(inv_temp), done)
    return bv, bi
