"""Attention operators: causal prefill over the fused qkv activation, paged decode.

``prefill_attention`` runs the tcgen05 flash kernel of ``csrc/attn_prefill.cu`` for bf16
with head_dim 128 (every Llama configuration here); other head sizes fall back to torch's
SDPA.  ``decode_attention`` runs the paged split-KV kernel of ``csrc/attn_decode.cu``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .._ext import ext

__all__ = ["prefill_attention", "decode_attention", "prefill_backend", "attn_status"]


def _native(qkv: torch.Tensor, hd: int) -> bool:
    return qkv.is_cuda and qkv.dtype == torch.bfloat16 and hd == 128


def prefill_backend(hd: int = 128) -> str:
    return "qfc-tcgen05" if hd == 128 else "sdpa"


def prefill_attention(qkv: torch.Tensor, B: int, S: int, nq: int, nkv: int, hd: int,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal self-attention of B sequences of length S; qkv [B*S, (nq+2nkv)*hd] -> [B*S, nq*hd]."""
    if _native(qkv, hd):
        o = torch.empty(B * S, nq * hd, dtype=qkv.dtype, device=qkv.device) if out is None else out
        ext().attn_prefill(qkv, o, B, S, nq, nkv, hd, 1.0 / hd ** 0.5)
        return o
    x = qkv.view(B, S, nq + 2 * nkv, hd)
    q = x[:, :, :nq].transpose(1, 2)
    k = x[:, :, nq:nq + nkv].transpose(1, 2)
    v = x[:, :, nq + nkv:].transpose(1, 2)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=(nq != nkv))
    o = o.transpose(1, 2).reshape(B * S, nq * hd)
    if out is not None:
        out.copy_(o)
        return out
    return o


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                     seq_lens: torch.Tensor, nq: int, nkv: int, hd: int,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per sequence over its paged cache.

    q [B, nq*hd]; caches [pages, nkv, page, hd]; block_table [B, max_pages] int32;
    seq_lens [B] int32 (tokens in the cache, including the current one).
    """
    o = torch.empty_like(q) if out is None else out
    ext().attn_decode(q, k_cache, v_cache, block_table, seq_lens, o, nq, nkv, hd, 1.0 / hd ** 0.5)
    return o


def attn_status(clear: bool = False) -> int:
    """Nonzero if the prefill attention kernel gave up waiting on a pipeline barrier."""
    return int(ext().attn_status(clear))
