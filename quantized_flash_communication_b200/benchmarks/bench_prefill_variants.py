"""The flagship prefill step under several all-reduce variants in one process.

    torchrun --nproc-per-node N -m quantized_flash_communication_b200.benchmarks.bench_prefill_variants \
        [--model llama2-7b --batch 8 --seq 1024] [--variants fused_sp,fused,unfused_sp,unfused,nccl]

One model (random-init N(0, 0.02) weights, synthetic token ids), one process group; for
every variant the step is captured as a CUDA graph and timed exactly like ``bench.py``
(warm-up, then CUDA events around --steps replays between barriers, maximum over ranks).
Variants:
  fused_sp    reduce-scatter fused into the o_proj / down_proj GEMM epilogues, and the
              sequence-parallel residual (all-reduce + residual + RMSNorm on the own rows)
  fused       GEMM-fused reduce-scatter, replicated residual + RMSNorm
  unfused_sp  GEMM, then the sequence-parallel all-reduce + norm kernel
  unfused     GEMM, then the all-reduce kernel, then RMSNorm on every row
  nccl        GEMM, then NCCL's bf16 all-reduce (the baseline), then RMSNorm
Rank 0 prints one JSON line per variant.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..communication import reset_communicators
from ..models.config import get_config
from ..models.llama import LlamaTP, TPContext
from ..utils.dist import init_distributed


def _max(x, dev):
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--bits", type=int, default=8)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--variants", default="fused_sp,fused,unfused_sp,unfused,nccl")
    args = ap.parse_args(argv)
    rank, world, dev = init_distributed()
    cfg = get_config(args.model)
    B, S = args.batch, args.seq
    tp = TPContext(None, dev, ar_backend="qfc", bits=args.bits, group_size=128, reserve_tokens=B * S,
                   hidden_size=cfg.hidden_size, seq_parallel=True)
    model = LlamaTP(cfg, tp, dev, init="shard", seed=1234)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(42)).to(dev)
    cache = model.new_cache(B, S)
    for name in args.variants.split(","):
        if world == 1 and name != "unfused":
            continue
        tp.ar_backend = "nccl" if name == "nccl" else "qfc"
        tp.fuse_gemm = name.startswith("fused")
        tp.fuse_max_world = 8 if tp.fuse_gemm else 0
        tp.seq_parallel = name.endswith("_sp")
        g = model.capture_prefill(B, S, cache)
        g.inp.copy_(ids)
        for _ in range(args.warmup):
            g()
        torch.cuda.synchronize()
        dist.barrier() if dist.is_initialized() else None
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            g()
        e.record()
        torch.cuda.synchronize()
        ms = _max(s.elapsed_time(e) / args.steps, dev)
        if tp.ar is not None:
            tp.ar.check()
        g.release()
        if rank == 0:
            print(json.dumps({"benchmark": "tp_prefill_variant", "variant": name, "model": cfg.name, "n_gpus": world,
                              "batch": B, "seq": S, "bits": args.bits, "ms_per_step": ms,
                              "tokens_per_s": B * S / (ms / 1000.0), "launch": "cuda_graph",
                              "data": "synthetic: uniform random token ids, random-init N(0,0.02) weights"}),
                  flush=True)
    reset_communicators()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
