"""tcgen05 GEMM throughput vs cuBLAS (torch.matmul) on the Llama-2-7B / Llama-3 shapes.

    python -m quantized_flash_communication_b200.benchmarks.bench_gemm [--shapes ...]
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops import gemm as G
from .timing import median, time_fn

# (name, M, N, K): prefill of 8 x 1024 tokens through Llama-2-7B layers at TP 1 and 8
SHAPES = [
    ("l2_7b_qkv_tp1", 8192, 12288, 4096),
    ("l2_7b_o_tp1", 8192, 4096, 4096),
    ("l2_7b_gateup_tp1", 8192, 22016, 4096),
    ("l2_7b_down_tp1", 8192, 4096, 11008),
    ("l2_7b_qkv_tp8", 8192, 1536, 4096),
    ("l2_7b_o_tp8", 8192, 4096, 512),
    ("l2_7b_gateup_tp8", 8192, 2752, 4096),
    ("l2_7b_down_tp8", 8192, 4096, 1376),
    ("square_8192", 8192, 8192, 8192),
]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default="")
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    rows = []
    for name, M, N, K in SHAPES:
        if args.only and args.only not in name:
            continue
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ours = median(time_fn(lambda: G.linear(a, b, out=out), args.iters))
        cub = median(time_fn(lambda: torch.matmul(a, b.T, out=out), args.iters))
        torch.cuda.synchronize()
        err = (G.linear(a, b).float() - (a.float() @ b.float().T)).abs().max().item()
        fl = 2.0 * M * N * K
        rows.append(dict(shape=name, M=M, N=N, K=K, ours_ms=ours, cublas_ms=cub,
                         ours_tflops=fl / ours / 1e9, cublas_tflops=fl / cub / 1e9, max_abs_err=err,
                         status=G.gemm_status()))
        print(json.dumps(rows[-1]), flush=True)
    return rows


if __name__ == "__main__":
    main()
