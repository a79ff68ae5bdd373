"""Attention operators: causal prefill over the fused qkv activation, paged decode.

``prefill_attention`` runs the hand-written sm_100a kernel when the extension provides
one (``_C.attn_prefill``); until then it uses torch's SDPA (flagged by
``PREFILL_BACKEND``).  ``decode_attention`` reads the paged KV cache.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .._ext import ext

__all__ = ["prefill_attention", "decode_attention", "prefill_backend"]


def prefill_backend() -> str:
    return "qfc" if hasattr(ext(), "attn_prefill") else "sdpa"


def prefill_attention(qkv: torch.Tensor, B: int, S: int, nq: int, nkv: int, hd: int,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal self-attention of B sequences of length S; qkv [B*S, (nq+2nkv)*hd] -> [B*S, nq*hd]."""
    C = ext()
    if hasattr(C, "attn_prefill"):
        o = torch.empty(B * S, nq * hd, dtype=qkv.dtype, device=qkv.device) if out is None else out
        C.attn_prefill(qkv, o, B, S, nq, nkv, hd, 1.0 / hd ** 0.5)
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
