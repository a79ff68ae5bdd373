"""All-reduce sweep: fused quantized all-reduce vs NCCL bf16.

    torchrun --nproc-per-node N -m quantized_flash_communication_b200.benchmarks.bench_allreduce \
        [--tokens 1,16,128,1024,4096,16384] [--hidden 4096,8192] [--bits 8,4] [--gs 32,64,128] [--reference]

Inputs: bf16 [tokens, hidden] drawn N(0,1) per rank with 0.1% outliers scaled x50.  For
every point: device time (CUDA events, median of --iters, maximum over ranks), NCCL-style
bus bandwidth of the equivalent bf16 all-reduce (2 (W-1)/W * bytes / time), relative L2
error against the exact fp32 sum, and the fraction of the NVLink roofline: the bytes this
rank must push over NVLink (two-shot: 2 (W-1)/W of the quantized payload; one-shot:
(W-1) x payload) at the measured 770 GB/s per direction, divided by the time.
``--reference`` also times the reference's flash_all_reduce (baseline/_ref, unmodified).
``--norm`` also times, for two-shot points with group 128, the all-reduce followed by the
residual add + RMSNorm on every row (the tensor-parallel layer's tail) against the
sequence-parallel kernel that does both on the rows each rank owns.
Rank 0 prints one JSON line per point.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

from ..communication import reset_communicators
from ..parallel.quant_allreduce import set_norm_warps_per_row, set_two_shot_stages
from ..parallel.quant_allreduce import QuantAllReduce
from ..quantization import rel_l2
from ..utils.dist import init_distributed

LINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200s


def _ints(s):
    return [int(x) for x in s.split(",") if x]


def _time(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    t = torch.tensor([ts[len(ts) // 2]], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _wire_bytes(n, W, bits, gs, one_shot):
    """Bytes one rank must push over NVLink (payload + fp16 scale/zero per group)."""
    from ..quantization import phase_bits

    def per_elem(p):
        return 2.0 if p == 16 else p / 8.0 + 4.0 / gs

    p1, p2 = phase_bits(bits)
    if one_shot:
        return (W - 1) * n * per_elem(8 if bits == 6 else p1)
    return (W - 1) / W * n * (per_elem(p1) + per_elem(p2))


def _norm_point(ar, xs, tokens, hidden, bits, rank, W, dev, iters, t_ar, wprs=(1,)):
    """all-reduce + residual RMSNorm of every row vs the sequence-parallel kernel (for each
    of ``wprs`` warps per row)."""
    from ..ops import layers as L
    eps = 1e-5
    w = torch.ones(hidden, dtype=torch.bfloat16, device=dev)
    h_full = torch.randn(tokens, hidden, device=dev).to(torch.bfloat16)
    R = (tokens + W - 1) // W
    h_shard = torch.zeros(R, hidden, dtype=torch.bfloat16, device=dev)
    n = max(0, min(tokens, (rank + 1) * R) - rank * R)
    h_shard[:n] = h_full[rank * R:rank * R + n]
    out = torch.empty_like(xs)
    x_out = torch.empty_like(xs)
    ar.reserve_rows(tokens, hidden, (bits,))

    def plain():
        ar(xs, out=out)
        L.rmsnorm(out, w, eps, residual=h_full, out=x_out)

    def fused():
        ar.all_reduce_norm(xs, h_shard, w, eps, out=x_out)

    t_plain = _time(plain, iters)
    for wpr in wprs:
        prev = set_norm_warps_per_row(wpr)
        t_sp = _time(fused, iters)
        set_norm_warps_per_row(prev)
        ar.check()
        if rank == 0:
            print(json.dumps({"impl": "allreduce_then_rmsnorm_vs_sequence_parallel", "W": W, "tokens": tokens,
                              "hidden": hidden, "bits": bits, "warps_per_row": wpr, "allreduce_ms": t_ar,
                              "allreduce_plus_rmsnorm_ms": t_plain, "allreduce_norm_sp_ms": t_sp,
                              "speedup": t_plain / t_sp}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,16,128,1024,4096,16384")
    ap.add_argument("--hidden", default="4096,8192")
    ap.add_argument("--bits", default="8,4")
    ap.add_argument("--gs", default="32,64,128")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--algo", default="auto")
    ap.add_argument("--reference", action="store_true")
    ap.add_argument("--norm", action="store_true")
    ap.add_argument("--norm-wpr", default="1", help="warps per row of the sequence-parallel kernel, e.g. 1,2,4")
    ap.add_argument("--stages", default="1", help="stages per CTA of the two-shot kernel, e.g. 1,2")
    args = ap.parse_args(argv)
    rank, W, dev = init_distributed()
    ar_cache = {}
    ref_far = None
    if args.reference:
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        sys.path.insert(0, os.path.join(root, "baseline", "_ref"))
        from communication import flash_all_reduce as ref_far  # noqa: E402  (reference, unmodified)
    for hidden in _ints(args.hidden):
        for tokens in _ints(args.tokens):
            n = tokens * hidden
            g = torch.Generator().manual_seed(1000 + rank)
            x = torch.randn(tokens, hidden, generator=g)
            x.view(-1)[torch.randperm(n, generator=g)[: max(1, n // 1000)]] *= 50
            xs = x.to(torch.bfloat16).to(dev)
            exact = xs.float().clone()
            dist.all_reduce(exact)
            buf = xs.clone()
            t_nccl = _time(lambda: dist.all_reduce(buf), args.iters)
            busbw = 2.0 * (W - 1) / W * n * 2 / (t_nccl * 1e-3) / 1e9
            rank0 = rank == 0
            if rank0:
                print(json.dumps({"impl": "nccl_bf16", "W": W, "tokens": tokens, "hidden": hidden,
                                  "ms": t_nccl, "busbw_gbs": busbw}), flush=True)
            for bits in _ints(args.bits):
                for gs in _ints(args.gs):
                    key = (bits, gs)
                    if key not in ar_cache:
                        ar_cache[key] = QuantAllReduce(None, dev, bits=bits, group_size=gs, algo=args.algo)
                    ar = ar_cache[key]
                    out = torch.empty_like(xs)
                    t = _time(lambda: ar(xs, out=out), args.iters)
                    ar.check()
                    err = rel_l2(out.float(), exact)
                    one = args.algo == "one_shot" or (args.algo == "auto" and n * 2 <= ar.one_shot_max_bytes)
                    wb = _wire_bytes(n, W, bits, gs, one)
                    roof_ms = wb / (LINK_GBS * 1e9) * 1e3
                    rec = {"impl": "qfc_fused", "W": W, "tokens": tokens, "hidden": hidden, "bits": bits, "gs": gs,
                           "algo": "one_shot" if one else "two_shot", "ms": t,
                           "busbw_gbs_equiv": 2.0 * (W - 1) / W * n * 2 / (t * 1e-3) / 1e9,
                           "speedup_vs_nccl": t_nccl / t, "rel_l2": err, "nvlink_bytes_per_rank": wb,
                           "roofline_ms": roof_ms, "roofline_frac": roof_ms / t}
                    for st in _ints(args.stages):
                        if st != 1 and not one:  # the staged kernel (two-shot only), same inputs
                            prev = set_two_shot_stages(st)
                            t_st = _time(lambda: ar(xs, out=out), args.iters)
                            set_two_shot_stages(prev)
                            ar.check()
                            rec[f"ms_stages{st}"] = t_st
                            rec[f"roofline_frac_stages{st}"] = roof_ms / t_st
                            rec[f"stages{st}_bit_exact"] = bool(torch.equal(out, ar(xs)))
                    if ref_far is not None:
                        xr = xs.to(torch.float16)
                        t_ref = _time(lambda: ref_far(xr.clone(), group_size=gs, bits=bits, quant_type="asym"),
                                      max(3, args.iters // 4))
                        yr, _ = ref_far(xr.clone(), group_size=gs, bits=bits, quant_type="asym")
                        rec["reference_ms"] = t_ref
                        rec["reference_rel_l2"] = rel_l2(yr.float(), exact)
                        rec["speedup_vs_reference"] = t_ref / t
                    if rank0:
                        print(json.dumps(rec), flush=True)
                    if args.norm and gs == 128 and not one and hidden % 256 == 0:
                        _norm_point(ar, xs, tokens, hidden, bits, rank, W, dev, args.iters, t,
                                    wprs=_ints(args.norm_wpr))
    reset_communicators()
    ar_cache.clear()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
