"""Run one kernel on a fixed small workload: the target of ``ncu`` captures and quick timings.

    python -m quantized_flash_communication_b200.benchmarks.kernel_probe gemm 8192 4096 4096
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe attention 8 1024 32 32
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe allreduce 2 16384 4096 8
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe allreduce_norm 2 8192 4096 8
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe quantize 67108864
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe decode 64 4096 16 4
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe rmsnorm 8192 4096
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe rope_decode 64 32 8
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe silu_mul 8192 11008
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe pack 67108864
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe unpack 67108864
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe oneshot 8 64 4096 8
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe gemm_qs8 8192 4096 4096
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe gemm_small 64 4096 14336
    python -m quantized_flash_communication_b200.benchmarks.kernel_probe qkv_rope 8192 4096 32 32

Switches of the opt-in kernels: --attn-packed (attention), --stages 2 (allreduce),
--norm-wpr 2|4|8 (allreduce_norm), --gemv (gemm / gemm_small with M <= 8).

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
    ap.add_argument("kernel", choices=["gemm", "attention", "allreduce", "allreduce_norm", "quantize", "decode",
                                       "rmsnorm", "rope_decode", "silu_mul", "pack", "unpack", "oneshot", "gemm_qs8",
                                       "gemm_small", "qkv_rope"])
    ap.add_argument("shape", nargs="*", type=int)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--attn-packed", action="store_true",
                    help="attention: the softmax with packed two-lane fp32 arithmetic")
    ap.add_argument("--stages", type=int, default=1, help="allreduce: stages per CTA of the two-shot kernel (1, 2)")
    ap.add_argument("--norm-wpr", type=int, default=1, help="allreduce_norm: warps per row (1, 2, 4, 8)")
    ap.add_argument("--gemv", action="store_true", help="gemm / gemm_small: the weight-streaming kernel (M <= 8)")
    args = ap.parse_args(argv)
    if args.attn_packed or args.stages != 1 or args.norm_wpr != 1 or args.gemv:
        from .._ext import ext
        ext().set_attn_packed(args.attn_packed)
        ext().set_two_shot_stages(args.stages)
        ext().set_norm_warps_per_row(args.norm_wpr)
        ext().set_gemv(args.gemv)
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
    elif args.kernel == "rmsnorm":
        from ..ops import layers as L
        M, H = args.shape or (8192, 4096)
        x = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
        r = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
        w = torch.ones(H, device=dev, dtype=torch.bfloat16)
        y = torch.empty_like(x)
        fn, work = (lambda: L.rmsnorm(x, w, 1e-5, residual=r, out=y)), float(M * H * 2 * 4)  # bytes: x, r in; r, y out
    elif args.kernel == "rope_decode":
        from ..ops import layers as L
        B, nq, nkv = args.shape or (64, 32, 8)
        hd, page, pps = 128, 64, 64
        qkv = torch.randn(B, (nq + 2 * nkv) * hd, device=dev, dtype=torch.bfloat16)
        cs = L.rope_cos_sin(8192, hd, 500000.0, dev)
        kc = torch.zeros(B * pps, nkv, page, hd, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        bt = torch.arange(B * pps, device=dev, dtype=torch.int32).view(B, pps)
        lens = torch.full((B,), 1000, device=dev, dtype=torch.int32)
        fn = lambda: L.rope_kv_decode(qkv, cs, nq, nkv, hd, kc, vc, bt, lens)  # noqa: E731
        work = float(qkv.numel() * 2 + B * nq * hd * 2 + 2 * B * nkv * hd * 2)  # bytes
    elif args.kernel == "silu_mul":
        from ..ops import layers as L
        M, I = args.shape or (8192, 11008)
        gu = torch.randn(M, 2 * I, device=dev, dtype=torch.bfloat16)
        y = torch.empty(M, I, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: L.silu_mul(gu, out=y)), float(M * I * 2 * 3)
    elif args.kernel in ("pack", "unpack"):
        from .. import kernels_jit as KJ
        (n,) = args.shape or (1 << 26,)
        codes = torch.randint(0, 16, (n,), device=dev, dtype=torch.int8)
        packed = KJ.pack_int4(codes)
        if args.kernel == "pack":
            fn, work = (lambda: KJ.pack_int4(codes)), float(n + n // 2)
        else:
            fn, work = (lambda: KJ.unpack_int4(packed, codes.shape)), float(n // 2 + n * 2)
    elif args.kernel == "oneshot":
        from ..parallel import EmulatedQuantAllReduce
        W, T, H, bits = args.shape or (8, 64, 4096, 8)
        ar = EmulatedQuantAllReduce(W, dev, bits=bits, group_size=128, algo="one_shot")
        xs = [torch.randn(T, H, device=dev, dtype=torch.bfloat16) for _ in range(W)]
        outs = [torch.empty_like(x) for x in xs]
        fn, work = (lambda: ar(xs, outs)), float(W * T * H)
    elif args.kernel == "gemm_qs8":
        from ..parallel import QuantAllReduce
        M, N, K = args.shape or (8192, 4096, 4096)
        ar = QuantAllReduce(None, dev, bits=8, group_size=128, algo="two_shot")  # one rank: own slots
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: ar.gemm_all_reduce(a, b, out=out)), 2.0 * M * N * K
    elif args.kernel == "gemm_small":
        from ..ops import gemm as G
        M, N, K = args.shape or (64, 4096, 14336)
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: G.linear(a, b, out=out)), float(N * K * 2)  # weight bytes streamed
    elif args.kernel == "qkv_rope":
        from ..ops import gemm as G
        from ..ops import layers as L
        M, K, nq, nkv = args.shape or (8192, 4096, 32, 32)
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        w = torch.randn((nq + 2 * nkv) * 128, K, device=dev, dtype=torch.bfloat16) * 0.02
        pos = torch.arange(M, device=dev) % 1024
        cs = L.rope_cos_sin(4096, 128, 10000.0, dev)
        out = torch.empty(M, w.shape[0], device=dev, dtype=torch.bfloat16)
        fn, work = (lambda: G.linear_qkv_rope(a, w, pos, cs, nq, nkv, out=out)), 2.0 * M * w.shape[0] * K
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
