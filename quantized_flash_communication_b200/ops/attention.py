"""Attention operators: causal prefill over the fused qkv activation, paged decode.

``prefill_attention`` runs the tcgen05 flash kernel of ``csrc/attn_prefill.cu``: bf16 on a
CUDA device with head_dim 128 (every Llama configuration here).  Any other input raises
instead of silently running a library kernel.  ``decode_attention`` runs the paged
split-KV kernel of ``csrc/attn_decode.cu``.
"""
from __future__ import annotations

import torch

from .._ext import ext

__all__ = ["prefill_attention", "decode_attention", "prefill_backend", "attn_status"]


def _native(qkv: torch.Tensor, hd: int) -> bool:
    return qkv.is_cuda and qkv.dtype == torch.bfloat16 and hd == 128


def prefill_backend(hd: int = 128) -> str:
    """Name of the kernel that serves prefill attention for head size ``hd``."""
    if hd != 128:
        raise ValueError(f"prefill attention has a kernel for head_dim 128 only, not {hd}")
    return "qfc-tcgen05"


def prefill_attention(qkv: torch.Tensor, B: int, S: int, nq: int, nkv: int, hd: int,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal self-attention of B sequences of length S; qkv [B*S, (nq+2nkv)*hd] -> [B*S, nq*hd]."""
    if not _native(qkv, hd):
        raise NotImplementedError(
            f"prefill_attention: the tcgen05 kernel takes bf16 CUDA tensors with head_dim 128; got "
            f"{qkv.dtype} on {qkv.device} with head_dim {hd}")
    o = torch.empty(B * S, nq * hd, dtype=qkv.dtype, device=qkv.device) if out is None else out
    ext().attn_prefill(qkv, o, B, S, nq, nkv, hd, 1.0 / hd ** 0.5)
    return o


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                     seq_lens: torch.Tensor, nq: int, nkv: int, hd: int,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per sequence over its paged cache.

    q [B, nq*hd] (rows may be strided, e.g. the q columns of the fused qkv activation);
    caches [pages, nkv, page, hd]; block_table [B, max_pages] int32; seq_lens [B] int32
    (tokens in the cache, including the current one).
    """
    o = torch.empty(q.shape[0], nq * hd, dtype=q.dtype, device=q.device) if out is None else out
    ext().attn_decode(q, k_cache, v_cache, block_table, seq_lens, o, nq, nkv, hd, 1.0 / hd ** 0.5)
    return o


def attn_status(clear: bool = False) -> int:
    """Nonzero if the prefill attention kernel gave up waiting on a pipeline barrier."""
    return int(ext().attn_status(clear))
