"""Rank-consistent token sampling for the tensor-parallel model.

The reference samples through Hugging Face ``generate(do_sample=True, temperature=0.7)``
with a wall-clock seed set on each rank (inference.py:24-36); the ranks agree only while
their seeds happen to coincide.  Here every rank draws the same token by construction:

* temperature sampling (``top_p == 1``) uses the Gumbel-max trick inside the argmax kernel
  (``csrc/layers.cu``): each rank adds Gumbel noise, keyed by (seed, step, row, global
  vocabulary index), to its slice of the vocabulary-parallel logits and the existing
  cross-rank argmax picks the winner.  The noise of a vocabulary entry does not depend on
  the rank or the tensor-parallel degree, so TP 1 and TP 8 draw the same token from the
  same logits;
* nucleus sampling (``top_p < 1``) gathers the full logits on every rank, keeps the
  smallest set of tokens whose probability reaches ``top_p`` and samples from it with the
  same Gumbel-max kernel over the whole vocabulary.

The seed is agreed once: rank 0 draws it (or takes the caller's) and broadcasts it.  The
step counter lives on the device and is advanced by the kernel, so a decode step captured
in a CUDA graph samples afresh on every replay.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from ..ops import layers as L

__all__ = ["Sampler", "top_p_mask"]


def top_p_mask(logits: torch.Tensor, inv_temp: float, top_p: float) -> torch.Tensor:
    """``logits`` with every token outside the top-p nucleus of softmax(logits * inv_temp)
    set to -inf (the smallest set whose probability reaches top_p; at least one token)."""
    scaled = logits.float() * inv_temp
    probs = torch.softmax(scaled, dim=-1)
    sp, order = probs.sort(dim=-1, descending=True)
    before = sp.cumsum(dim=-1) - sp           # probability of the tokens ranked above
    drop_sorted = before >= top_p
    drop_sorted[..., 0] = False
    drop = torch.zeros_like(drop_sorted).scatter_(-1, order, drop_sorted)
    return logits.float().masked_fill(drop, float("-inf"))


class Sampler:
    """Sampling state of one model replica group: seed and step on the device."""

    def __init__(self, tp, temperature: float = 1.0, top_p: float = 1.0, seed: Optional[int] = None):
        if temperature <= 0:
            raise ValueError("temperature must be > 0 (use greedy decoding for temperature 0)")
        if not 0.0 < top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        self.tp = tp
        self.inv_temp = 1.0 / temperature
        self.top_p = top_p
        dev = tp.device
        if seed is None:
            seed = int.from_bytes(os.urandom(8), "little") & ((1 << 62) - 1)
        state = torch.tensor([seed, 0], dtype=torch.int64, device=dev)
        if tp.world > 1:  # every rank uses rank 0's seed
            dist.broadcast(state, src=dist.get_global_rank(tp.group, 0) if tp.group is not None else 0,
                           group=tp.group)
        self.state = state                      # [seed, step]; the kernel advances step
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)  # the kernel's arrival counter

    @property
    def seed(self) -> int:
        return int(self.state[0].item())

    def local(self, logits: torch.Tensor, vocab_start: int, valid: int):
        """(score, global index) of this rank's best sampled candidate per row, for the
        temperature-only path (the caller combines ranks with its argmax gather)."""
        return L.argmax(logits, vocab_start, valid=valid, rng=self.state, inv_temp=self.inv_temp, done=self.done)

    def full(self, logits: torch.Tensor) -> torch.Tensor:
        """Token per row from the full-vocabulary logits (identical on every rank)."""
        if self.top_p < 1.0:
            logits = top_p_mask(logits, self.inv_temp, self.top_p)
        _, idx = L.argmax(logits.contiguous(), 0, rng=self.state, inv_temp=self.inv_temp, done=self.done)
        return idx
