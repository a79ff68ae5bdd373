"""Run one kernel on a fixed small workload: the target of ``ncu`` captures and quick timings.

    python -m quantized_flash_communication_b200.benchmarks.kernel_probe gemm 8192 4096 4096
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe attention 8 1024 32 32
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe allreduce 2 16384 4096 8
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe allreduce_norm 2 8192 4096 8
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe quantize 67108864
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe decode 64 4096 16 4

Each subcommand runs ``--iters`` launches (default 3) after one warm-up and prints the
median device time; ``allreduce`` and ``allreduce_norm`` (the sequence-parallel
all-reduce + residual + RMSNorm) run W ranks emulated inside one launch on one GPU.
"""
from __future__ import annotations

import argparse
import json

import torch

from .timing import median, time_fn


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemm", "attention", "allreduce", "allreduce_norm", "quantize", "decode"])
    ap.add_argument("shape", nargs="*", type=int)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    if args.kernel == "gemm":
        from ..ops import gemm as G
        M, N, K = args.shape or (8192, 4096, 4096)
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: G.linear(a, b, out=out)), 2.0 * M * N * K
    elif args.kernel == "attention":
        from ..ops import attention as A
        B, S, nq, nkv = args.shape or (8, 1024, 32, 32)
        qkv = torch.randn(B * S, (nq + 2 * nkv) * 128, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: A.prefill_attention(qkv, B, S, nq, nkv, 128)), 2.0 * B * nq * S * S * 128
    elif args.kernel == "allreduce":
        from ..parallel import EmulatedQuantAllReduce
        W, T, H, bits = args.shape or (2, 16384, 4096, 8)
        ar = EmulatedQuantAllReduce(W, dev, bits=bits, group_size=128, algo="two_shot")
        xs = [torch.randn(T, H, device=dev, dtype=torch.bfloat16) for _ in range(W)]
        outs = [torch.empty_like(x) for x in xs]
        fn, work = (lambda: ar(xs, outs)), float(W * T * H)
    elif args.kernel == "allreduce_norm":
        from ..parallel import EmulatedQuantAllReduce
        W, T, H, bits = args.shape or (2, 8192, 4096, 8)
        ar = EmulatedQuantAllReduce(W, dev, bits=bits, group_size=128, algo="two_shot")
        R = (T + W - 1) // W
        xs = [torch.randn(T, H, device=dev, dtype=torch.bfloat16) for _ in range(W)]
        hs = [torch.randn(R, H, device=dev, dtype=torch.bfloat16) for _ in range(W)]
        w = torch.ones(H, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: ar.all_reduce_norm(xs, hs, w, 1e-5)), float(W * T * H)
    elif args.kernel == "quantize":
        from ..ops import quant as Q
        (n,) = args.shape or (1 << 26,)
        x = torch.randn(n, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: Q.quantize(x, 8, 128)), float(n)
    else:
        from ..ops.attention import decode_attention
        B, ctx, nq, nkv = args.shape or (64, 4096, 16, 4)
        page = 64
        pps = (ctx + page - 1) // page
        kc = torch.randn(B * pps, nkv, page, 128, device=dev, dtype=torch.bfloat16)
        vc = torch.randn_like(kc)
        bt = torch.arange(B * pps, device=dev, dtype=torch.int32).view(B, pps)
        lens = torch.full((B,), ctx, device=dev, dtype=torch.int32)
        q = torch.randn(B, nq * 128, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: decode_attention(q, kc, vc, bt, lens, nq, nkv, 128)), float(B * ctx * nkv * 128 * 4)
    ms = median(time_fn(fn, iters=args.iters, warmup=1, flush=False))
    print(json.dumps({"kernel": args.kernel, "shape": args.shape, "ms": ms, "work_per_ms": work / ms}))


if __name__ == "__main__":
    main()
