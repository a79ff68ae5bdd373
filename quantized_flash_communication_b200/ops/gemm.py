"""tcgen05 / TMEM GEMM (``csrc/gemm.cu``): ``a @ b.T`` with fused epilogues.

Replaces the cuBLAS GEMMs behind the reference's ``nn.Linear`` layers (model.py:32-35).
"""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import ext

__all__ = ["linear", "linear_swiglu", "linear_residual", "linear_qkv_rope", "gemm_status", "EPI_STORE", "EPI_SWIGLU",
           "EPI_RESIDUAL"]

EPI_STORE, EPI_SWIGLU, EPI_RESIDUAL = 0, 1, 2


def _2d(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, x.shape[-1])


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ w.T`` for bf16 ``x [..., K]`` and ``w [N, K]``."""
    y = ext().gemm_bf16(_2d(x), w, None if out is None else _2d(out), EPI_STORE)
    return y.view(*x.shape[:-1], w.shape[0])


def linear_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(x @ gate.T) * (x @ up.T)`` for ``w_gate_up = [gate; up]`` of shape [2I, K]."""
    I = w_gate_up.shape[0] // 2
    y = ext().gemm_bf16(_2d(x), w_gate_up, None if out is None else _2d(out), EPI_SWIGLU)
    return y.view(*x.shape[:-1], I)


def linear_residual(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ w.T + residual`` (``out`` may alias ``residual``)."""
    y = ext().gemm_bf16(_2d(x), w, None if out is None else _2d(out), EPI_RESIDUAL, _2d(residual))
    return y.view(*x.shape[:-1], w.shape[0])


def linear_qkv_rope(x: torch.Tensor, w_qkv: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor, nq: int, nkv: int,
                    k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None,
                    slots: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ w_qkv.T`` with the rotary embedding of its q and k heads applied at ``pos`` and
    its k, v heads written to the paged caches at ``slots``, all in the GEMM's epilogue
    (head_dim 128).  Same result as :func:`linear` followed by ``layers.rope_kv``."""
    x2 = _2d(x)
    y = torch.empty(x2.shape[0], w_qkv.shape[0], dtype=x.dtype, device=x.device) if out is None else _2d(out)
    ext().gemm_qkv_rope(x2, w_qkv, y, pos, cos_sin, k_cache, v_cache, slots, nq, nkv)
    return y.view(*x.shape[:-1], w_qkv.shape[0])


def gemm_status(clear: bool = False) -> int:
    """Nonzero if a GEMM kernel gave up waiting on one of its pipeline barriers."""
    return int(ext().gemm_status(clear))
