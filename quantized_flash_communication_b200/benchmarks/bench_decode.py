"""Prefill + decode benchmark (Llama-3-8B at TP 2/4/8, Llama-3-70B at TP 8).

    torchrun --nproc-per-node N -m quantized_flash_communication_b200.benchmarks.bench_decode \
        --model llama3-8b --batch 64 --ctx 4096 --new 128 --bits 8
    torchrun --nproc-per-node 8 -m quantized_flash_communication_b200.benchmarks.bench_decode \
        --model llama3-70b --batch 4 --ctx 2048 --new 128 --bits 4

Random-init weights N(0, 0.02), uniformly random token ids.  The context is prefilled
(timed: TTFT, CUDA events, max over ranks); then each decode step (one token for every
sequence, one CUDA graph replay that includes the quantized all-reduces and the argmax
combine) is timed over ``new - 1`` steps after ``--warmup`` untimed steps.  Rank 0 prints one
JSON line: TTFT, per-token latency and decode tokens/s for the whole batch.

``--impl reference`` times the reference's own path on the same shapes: Hugging Face
``generate`` (the call of the reference's QA test, inference.py:29-36) on a random-init
``LlamaForCausalLM`` with the reference's injected tensor-parallel MLPs and its
``flash_all_reduce`` (benchmarks/reference_arm.py), greedy, fp16.  TTFT is a
``generate`` of one token; the per-token latency is (a ``generate`` of ``new`` tokens minus
TTFT) / (new - 1), both CUDA-event timed, max over ranks.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..communication import reset_communicators
from ..models.config import get_config
from ..models.llama import LlamaTP, TPContext
from ..utils.clocks import ClockSampler
from ..utils.dist import init_distributed


def _max(x: float, dev) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def _run_reference(args, cfg, rank, world, dev):
    from .reference_arm import build_reference_model, reference_available
    if not reference_available():
        if rank == 0:
            print(json.dumps({"benchmark": "tp_decode", "impl": "reference", "unavailable": "baseline/_ref is missing"}))
        return
    if not dist.is_initialized():  # the reference's all-reduce needs a process group, also for one rank
        import os
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29541")
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev)
    B, S = args.batch, args.ctx
    model = build_reference_model(cfg, dev, rank, world, bits=args.bits, group_size=args.group_size)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(1)).to(dev)
    mask = torch.ones_like(ids)

    def gen(n):
        with torch.no_grad():
            return model.generate(ids, attention_mask=mask, max_new_tokens=n, min_new_tokens=n, do_sample=False,
                                  pad_token_id=0)

    gen(2)  # warm-up: the reference's Triton / JIT kernels compile here
    torch.cuda.synchronize()
    _barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    gen(1)
    e.record()
    torch.cuda.synchronize()
    ttft = _max(s.elapsed_time(e), dev)
    _barrier()
    sampler = ClockSampler(list(range(world)) if world > 1 else [dev.index]) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    s.record()
    out = gen(args.new)
    e.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__(None, None, None)
    total = _max(s.elapsed_time(e), dev)
    per_tok = (total - ttft) / max(1, args.new - 1)
    if rank == 0:
        print(json.dumps({
            "benchmark": "tp_decode", "impl": "reference", "model": cfg.name, "n_gpus": world, "batch": B, "ctx": S,
            "new_tokens": args.new, "generated": int(out.shape[1] - S),
            "allreduce": f"reference flash_all_reduce INT{args.bits} g{args.group_size} asym (MLP only)",
            "ttft_ms": ttft, "per_token_ms": per_tok, "decode_tokens_per_s": B * 1000.0 / per_tok, "dtype": "fp16",
            "api": "transformers generate (greedy) + reference inject_ultimate_layers + flash_all_reduce",
            "clocks": sampler.summary() if sampler else None,
            "data": "synthetic: uniform random token ids, random-init N(0,0.02) weights"}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--bits", type=int, default=8)
    ap.add_argument("--group-size", type=int, default=128)
    ap.add_argument("--ar-backend", default="qfc", choices=["qfc", "nccl"])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (debug only)")
    ap.add_argument("--breakdown", action="store_true",
                    help="also time eager decode steps per operator (CUDA-event regions, max over ranks)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--gemv", action="store_true",
                    help="GEMMs of at most 8 rows on the weight-streaming kernel (set_gemv)")
    args = ap.parse_args(argv)
    if args.gemv and args.impl == "ours":
        from .._ext import ext
        ext().set_gemv(True)
    rank, world, dev = init_distributed()
    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.with_layers(args.layers)
    if args.impl == "reference":
        _run_reference(args, cfg, rank, world, dev)
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()
        return
    B, S = args.batch, args.ctx
    tp = TPContext(None, dev, ar_backend=args.ar_backend, bits=args.bits, group_size=args.group_size,
                   reserve_tokens=B * S, hidden_size=cfg.hidden_size)
    model = LlamaTP(cfg, tp, dev, init="shard", seed=7)
    cache = model.new_cache(B, S + args.new + args.warmup + 1 + (8 if args.breakdown else 0))
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(1)).to(dev)
    model.prefill(ids, cache)  # warm-up (JIT-free kernels; sizes the workspaces)
    torch.cuda.synchronize()
    _barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    tok = model.prefill(ids, cache)
    e.record()
    torch.cuda.synchronize()
    ttft = _max(s.elapsed_time(e), dev)

    step = model.capture_decode(cache)
    cur = tok
    for _ in range(args.warmup):
        cur = step(cur).clone()
    torch.cuda.synchronize()
    _barrier()
    n = max(1, args.new - 1)
    sampler = ClockSampler(list(range(world)) if world > 1 else [dev.index]) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    s.record()
    for _ in range(n):
        cur = step(cur)
    e.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__(None, None, None)
    per_tok = _max(s.elapsed_time(e), dev) / n
    if tp.ar is not None:
        tp.ar.check()
    step.release()
    breakdown = None
    if args.breakdown:
        from ..utils.trace import OpTimer
        timer = OpTimer()
        model.timer = tp.timer = timer
        for _ in range(4):
            cur = model.decode_step(cur, cache)
        summ = timer.summary()
        model.timer = tp.timer = None
        names = list(summ)
        vals = torch.tensor([summ[k]["ms"] / 4 for k in names], dtype=torch.float64, device=dev)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        breakdown = {k: round(float(v), 4) for k, v in zip(names, vals.tolist())}
    if rank == 0:
        print(json.dumps({
            "benchmark": "tp_decode", "model": cfg.name, "n_gpus": world, "batch": B, "ctx": S, "new_tokens": args.new,
            "allreduce": f"{args.ar_backend} INT{args.bits} g{args.group_size}" if world > 1 else "none (tp1)",
            "ttft_ms": ttft, "per_token_ms": per_tok, "decode_tokens_per_s": B * 1000.0 / per_tok,
            "launch": "cuda_graph", "small_m_gemm": "weight-streaming (gemv)" if args.gemv else "tcgen05",
            "clocks": sampler.summary() if sampler else None,
            "eager_breakdown_ms_per_token": breakdown,
            "data": "synthetic: uniform random token ids, random-init N(0,0.02) weights"}), flush=True)
    reset_communicators()
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
