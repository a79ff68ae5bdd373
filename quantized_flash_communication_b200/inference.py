"""Reference-compatible generation test (reference inference.py:4-46).

``run_qa_test(model, tokenizer, device, rank)`` switches every all-reduce of the
tensor-parallel model to the flash INT6 mode (INT4 reduce-scatter + INT8 all-gather, as the
reference does at inference.py:9-12), generates ``max_new_tokens`` tokens for a prompt and
reports the wall time on rank 0.  Like the reference (inference.py:29-36) it samples with
temperature 0.7 by default (``do_sample=False`` decodes greedily).  The reference seeds each
rank with the wall clock (inference.py:24) and relies on the seeds coinciding; here rank 0
picks the seed and broadcasts it, and the sampler draws the same token on every rank by
construction (``models/sampling.py``).  Without a tokenizer the prompt is mapped to token
ids byte by byte.
"""
from __future__ import annotations

import time
from typing import Optional, Tuple

import torch

__all__ = ["run_qa_test", "encode_prompt"]


def encode_prompt(prompt: str, vocab_size: int, tokenizer=None) -> list:
    if tokenizer is not None:
        return list(tokenizer.encode(prompt))
    return [b % vocab_size for b in prompt.encode("utf-8")]


@torch.no_grad()
def run_qa_test(model, tokenizer=None, device=None, rank: Optional[int] = None, prompt: str = "Explain london.",
                max_new_tokens: int = 200, bits: int = 6, group_size: int = 128, quant_type: str = "asym",
                verbose: bool = True, do_sample: bool = True, temperature: float = 0.7, top_p: float = 1.0,
                seed: Optional[int] = None) -> Tuple[torch.Tensor, float]:
    """Generate with the flash all-reduce; returns (new token ids [1, n], total ms).

    ``top_p`` defaults to 1 (Hugging Face's default when a checkpoint has no generation
    config; Llama-3.2-3B-Instruct's own generation config sets 0.9)."""
    device = torch.device(device) if device is not None else model.device
    rank = model.tp.rank if rank is None else rank
    model.tp.configure(bits=bits, group_size=group_size, quant_type=quant_type,
                       backend="qfc" if model.tp.world > 1 else None)
    ids = torch.tensor([encode_prompt(prompt, model.cfg.vocab_size, tokenizer)], dtype=torch.int64, device=device)
    if verbose and rank == 0:
        print(f"[QA test] prompt: {prompt}")
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    out = model.generate(ids, max_new_tokens, do_sample=do_sample, temperature=temperature, top_p=top_p, seed=seed)
    torch.cuda.synchronize(device)
    total_ms = (time.perf_counter() - t0) * 1000.0
    if verbose and rank == 0:
        toks = out[0].tolist()
        text = tokenizer.decode(toks, skip_special_tokens=True) if tokenizer is not None else str(toks[:32])
        print(f"[QA test] answer: {text}")
        print(f"[QA test] total generation time: {total_ms:.2f} ms for {max_new_tokens} tokens")
    return out, total_ms
