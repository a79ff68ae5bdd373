"""Flagship benchmark: tensor-parallel Llama-2-7B prefill (TTFT) on N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

The flagship configuration: Llama-2-7B architecture (32 layers, hidden 4096, 32 heads, SwiGLU
11008, vocab 32000), bf16 random-init N(0, 0.02) weights, batch 8 x 1024 uniformly random
token ids, an INT8 (group 128) quantized all-reduce after o_proj and down_proj.  One step
is one prefill of the whole batch up to the first generated token (TTFT); ``value`` is
the job's prefill throughput in tokens/s (batch * seq / TTFT).  Timing: W untimed steps,
then K steps between a barrier + synchronize on both sides, CUDA events on the
launching stream, maximum over ranks.

``--impl reference`` runs the unmodified reference (baseline/_ref): Hugging Face
LlamaForCausalLM with the same architecture and init, the reference's
``inject_ultimate_layers`` (MLP-only tensor parallelism) and its ``flash_all_reduce``
in INT8 / group 128 / asym mode, in fp16 (its all-reduce always returns fp16).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
import types

ROOT = os.path.dirname(os.path.abspath(__file__))


def _parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--bits", type=int, default=8)
    ap.add_argument("--group-size", type=int, default=128)
    ap.add_argument("--quant-type", default="asym")
    ap.add_argument("--ar-backend", default="qfc", choices=["qfc", "nccl", "staged"])
    ap.add_argument("--e2e-steps", type=int, default=None, help="host-timed end-to-end steps (default: --steps)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch kernels eagerly instead of one CUDA graph")
    ap.add_argument("--seq-parallel", action="store_true",
                    help="sequence-parallel residual stream at every world size (the default turns it on from 2 ranks)")
    ap.add_argument("--breakdown", action="store_true",
                    help="print per-operator device times of eager steps instead of the benchmark line")
    ap.add_argument("--no-fuse-gemm", action="store_true",
                    help="run o_proj/down_proj GEMMs and the all-reduce as separate kernels")
    return ap.parse_args()


def _dist_init(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1 or args.impl == "reference":
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        os.environ.setdefault("RANK", str(rank))
        os.environ.setdefault("WORLD_SIZE", str(world))
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=600),
                                device_id=dev)
    return rank, world, dev


def _max_over_ranks(x: float, dev) -> float:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def _timed(step_fn, args, dev, rank, world):
    """Warm up, then time K steps on the device (events), max over ranks."""
    import torch
    from quantized_flash_communication_b200.utils.clocks import ClockSampler
    for _ in range(args.warmup):
        step_fn()
    torch.cuda.synchronize()
    _barrier()
    torch.cuda.synchronize()
    gpus = list(range(world)) if world > 1 else [dev.index]
    sampler = ClockSampler(gpus) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        step_fn()
    e.record()
    torch.cuda.synchronize()
    _barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__(None, None, None)
    ms = _max_over_ranks(s.elapsed_time(e), dev) / args.steps
    return ms, (sampler.summary() if sampler else None)


def _timed_e2e(step_fn, args, dev):
    """Host-timed steps that include the pinned H2D input copy and the D2H result read
    (as many as the device-timed steps unless --e2e-steps says otherwise)."""
    import torch
    n = args.e2e_steps or args.steps
    for _ in range(max(1, args.warmup)):
        step_fn()
    torch.cuda.synchronize()
    _barrier()
    t0 = time.perf_counter()
    for _ in range(n):
        step_fn()
    t1 = time.perf_counter()
    _barrier()
    return _max_over_ranks((t1 - t0) * 1000.0 / n, dev)


def _peaks():
    """Roofline denominators: the driver-measured peaks if present, else the pool's fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops_sustained"]), float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1400.0, 6650.0, "fallback"


LINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200s


def _step_flops(cfg, B, S):
    """FLOPs of one prefill step of the whole model: the linear layers over every token,
    causal attention, and the lm_head over the last token of each sequence."""
    H, hd = cfg.hidden_size, cfg.head_dim
    qkv = H * (cfg.num_heads + 2 * cfg.num_kv_heads) * hd
    per_layer = 2 * B * S * (qkv + cfg.num_heads * hd * H + 3 * H * cfg.intermediate_size)
    per_layer += 2 * B * cfg.num_heads * S * S * hd  # QK^T and PV, causal half of each
    return cfg.num_layers * per_layer + 2 * B * H * cfg.vocab_size


def _wire_bytes_per_step(cfg, B, S, W, bits, gs):
    """Bytes one rank pushes over NVLink per step: two two-shot all-reduces per layer of
    [B*S, H], each 2 (W-1)/W of the quantized payload plus fp16 (scale, zero) per group."""
    if W == 1:
        return 0.0
    from quantized_flash_communication_b200.quantization import phase_bits
    p1, p2 = phase_bits(bits)

    def per_elem(p):
        return 2.0 if p == 16 else p / 8.0 + 4.0 / gs
    n = B * S * cfg.hidden_size
    return cfg.num_layers * 2 * (W - 1) / W * n * (per_elem(p1) + per_elem(p2))


def _quant_error(model, tp, ids, dev):
    """Relative L2 error of one step's all-reduce against the exact fp32 sum.

    Runs layer 0 of a real step up to o_proj on this rank, forms its partial sum, and
    all-reduces it twice: through the model's quantized path and exactly in fp32 (NCCL,
    outside any timed region).  The fused GEMM epilogue is bit-identical to this unfused
    pair, so the error is that of the step's all-reduces."""
    import torch
    import torch.distributed as dist
    from quantized_flash_communication_b200.ops import attention as A
    from quantized_flash_communication_b200.ops import gemm as G
    from quantized_flash_communication_b200.ops import layers as L
    from quantized_flash_communication_b200.quantization import rel_l2
    if tp.world == 1 or tp.ar is None:
        return None
    cfg = model.cfg
    B, S = ids.shape
    lay = model.model.layers[0]
    h = L.embedding(ids.reshape(-1), model.model.embed_tokens.weight)
    x = L.rmsnorm(h, lay.input_layernorm.weight, cfg.rms_eps)
    qkv = G.linear(x, lay.self_attn.qkv_fused)
    pos = torch.arange(S, device=dev, dtype=torch.int64).repeat(B)
    L.rope_kv(qkv, pos, model.cos_sin, model.nq, model.nkv, model.hd, None, None, None)
    o = A.prefill_attention(qkv, B, S, model.nq, model.nkv, model.hd)
    p = G.linear(o, lay.self_attn.o_proj.weight)
    exact = p.float()
    dist.all_reduce(exact)
    got = tp.all_reduce(p.clone())
    torch.cuda.synchronize()
    err = torch.tensor([rel_l2(got.float(), exact)], device=dev, dtype=torch.float64)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    return float(err.item())


# ------------------------------------------------------------------------------------------
def _breakdown(args, model, tp, ids, cache, dev, rank, world):
    """Eager steps with per-operator CUDA-event regions; prints max-over-ranks totals."""
    import torch
    import torch.distributed as dist
    from quantized_flash_communication_b200.utils.trace import OpTimer

    for _ in range(args.warmup):
        model.prefill(ids, cache)
    timer = OpTimer()
    model.timer = tp.timer = timer
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        model.prefill(ids, cache)
    e.record()
    summ = timer.summary()
    model.timer = tp.timer = None
    names = list(summ.keys())
    vals = torch.tensor([summ[n]["ms"] / args.steps for n in names] + [s.elapsed_time(e) / args.steps],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    if rank == 0:
        from quantized_flash_communication_b200.benchmarks.roofline import fractions, op_bounds
        out = {n: round(float(v), 4) for n, v in zip(names, vals[:-1].tolist())}
        counts = {n: summ[n]["count"] // args.steps for n in names}
        peak_tf, hbm_gbs, peak_src = _peaks()
        B, S = ids.shape
        bounds = op_bounds(model.cfg, B, S, world, args.bits, args.group_size, peak_tf, hbm_gbs)
        print(json.dumps({"breakdown_ms_per_step_max_over_ranks": out, "eager_ms_per_step": float(vals[-1]),
                          "n_gpus": world, "fuse_gemm": not args.no_fuse_gemm, "ar_backend": args.ar_backend,
                          "counts_per_step": counts,
                          "roofline_per_region": fractions(out, counts, bounds),
                          "roofline_peaks": f"{peak_src}: {peak_tf} TFLOP/s bf16 sustained, {hbm_gbs} GB/s copy, "
                                            "770 GB/s NVLink per direction"}), flush=True)
    return None


def run_ours(args):
    import torch
    sys.path.insert(0, ROOT)
    from quantized_flash_communication_b200._ext import count_launches
    from quantized_flash_communication_b200.models.config import get_config
    from quantized_flash_communication_b200.models.llama import LlamaTP, TPContext
    from quantized_flash_communication_b200.ops import attention as A
    from quantized_flash_communication_b200.ops.gemm import gemm_status

    rank, world, dev = _dist_init(args)
    cfg = get_config(args.model)
    B, S = args.batch, args.seq
    tp = TPContext(None, dev, ar_backend=args.ar_backend, bits=args.bits, group_size=args.group_size,
                   quant_type=args.quant_type, algo="auto", reserve_tokens=B * S, hidden_size=cfg.hidden_size,
                   fuse_gemm=not args.no_fuse_gemm, seq_parallel=args.seq_parallel or None)
    model = LlamaTP(cfg, tp, dev, init="shard", seed=1234)
    g = torch.Generator(device="cpu").manual_seed(42)
    ids_host = torch.randint(0, cfg.vocab_size, (B, S), generator=g).pin_memory()
    ids = ids_host.to(dev)
    cache = model.new_cache(B, S)
    with count_launches() as cnt:  # one eager step: which of our kernels a step launches
        model.prefill(ids, cache)
    torch.cuda.synchronize()
    launches_per_step = cnt["kernels"]
    if args.breakdown:
        _breakdown(args, model, tp, ids, cache, dev, rank, world)
        return rank, None
    graphed = None
    if not args.no_graph:
        graphed = model.capture_prefill(B, S, cache)
        graphed.inp.copy_(ids)

        def step():
            return graphed()
    else:
        def step():
            return model.prefill(ids, cache)

    ms, clocks = _timed(step, args, dev, rank, world)
    torch.cuda.synchronize()
    if tp.ar is not None:
        tp.ar.check()
    assert gemm_status() == 0, "a GEMM kernel reported a pipeline timeout"
    qerr = _quant_error(model, tp, ids, dev) if args.ar_backend == "qfc" else None

    e2e = None
    if not args.no_e2e:
        out_host = torch.empty(B, dtype=torch.int64).pin_memory()

        def e2e_step():
            if graphed is not None:
                graphed.inp.copy_(ids_host, non_blocking=True)  # pinned host -> device
                nxt = graphed()
            else:
                nxt = model.prefill(ids_host.to(dev, non_blocking=True), cache)
            out_host.copy_(nxt, non_blocking=True)  # device -> pinned host
            torch.cuda.current_stream().synchronize()
            return out_host

        e2e_ms = _timed_e2e(e2e_step, args, dev)
        e2e = {"value": B * S / (e2e_ms / 1000.0), "unit": "tokens/s", "ttft_ms": e2e_ms,
               "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(),
               "d2h_bytes_per_step": out_host.numel() * out_host.element_size(),
               "api": "LlamaTP.capture_prefill (CUDA graph)" if graphed is not None else "LlamaTP.prefill"}
    weights_gb = sum(p.numel() * p.element_size() for p in model.parameters()) / 1e9
    peak_tf, _, peak_src = _peaks()
    flops = _step_flops(cfg, B, S)
    wire = _wire_bytes_per_step(cfg, B, S, world, args.bits, args.group_size) if args.ar_backend == "qfc" else 0.0
    t_compute = flops / world / (peak_tf * 1e12) * 1e3
    t_link = wire / (LINK_GBS * 1e9) * 1e3
    roofline = {"fraction": max(t_compute, t_link) / ms, "compute_ms_at_peak": t_compute,
                "nvlink_ms_at_770gbs": t_link, "flops_per_step": flops, "nvlink_bytes_per_rank": wire,
                "peak_tflops": peak_tf, "peaks": f"{peak_src} (bf16 sustained)",
                "note": "the slower of compute at peak and bytes over NVLink, divided by the step time"}
    res = {
        "metric": "tp_prefill_throughput_llama2_7b",
        "value": B * S / (ms / 1000.0),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "ttft_ms": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: uniform random token ids, random-init N(0,0.02) weights",
        "config": {"model": cfg.name, "global_batch": B, "seq_len": S, "parallelism": f"tp{world}",
                   "allreduce": (f"qfc INT{args.bits} g{args.group_size} {args.quant_type}"
                                 + (", scatter fused into o/down GEMM epilogues"
                                    if tp.fuse_gemm and world <= tp.fuse_max_world else "")
                                 + (", sequence-parallel residual + RMSNorm in the all-reduce"
                                    if tp.sp_active(B * S, cfg.hidden_size) else "")
                                 if args.ar_backend == "qfc" else args.ar_backend) if world > 1 else "none (tp1)",
                   "attention": A.prefill_backend(cfg.head_dim),
                   "launch": "cuda_graph" if graphed is not None else "eager",
                   "l2": f"no flush; each step streams {weights_gb:.1f} GB of weights per rank (> 126 MB L2)"},
        "clocks": clocks,
        "e2e": e2e,
        "roofline_fraction": roofline["fraction"],
        "roofline": roofline,
        "quant_rel_l2": qerr,
        "gpu_launches": launches_per_step * args.steps,
        "gpu_launches_per_step": launches_per_step,
        "impl": "ours",
    }
    if graphed is not None:
        graphed.release()
    return rank, res


# ------------------------------------------------------------------------------------------
def run_reference(args):
    import torch
    sys.path.insert(0, ROOT)
    from quantized_flash_communication_b200.benchmarks.reference_arm import build_reference_model, reference_available
    if not reference_available():
        return 0, {"impl": "reference", "unavailable": "baseline/_ref is missing (copy the reference's 7 .py files)"}
    rank, world, dev = _dist_init(args)
    from quantized_flash_communication_b200.models.config import get_config
    cfg = get_config(args.model)
    model = build_reference_model(cfg, dev, rank, world, args.bits, args.group_size, args.quant_type)
    B, S = args.batch, args.seq
    g = torch.Generator(device="cpu").manual_seed(42)
    ids_host = torch.randint(0, cfg.vocab_size, (B, S), generator=g).pin_memory()
    ids = ids_host.to(dev)

    def step():
        with torch.no_grad():
            return model(ids).logits

    ms, clocks = _timed(step, args, dev, rank, world)
    e2e = None
    if not args.no_e2e:
        def e2e_step():
            d = ids_host.to(dev, non_blocking=True)
            with torch.no_grad():
                nxt = model(d).logits[:, -1].argmax(-1)
            return nxt.cpu()
        e2e_ms = _timed_e2e(e2e_step, args, dev)
        e2e = {"value": B * S / (e2e_ms / 1000.0), "unit": "tokens/s", "ttft_ms": e2e_ms,
               "h2d_bytes_per_step": ids_host.numel() * 8, "d2h_bytes_per_step": B * 8,
               "api": "reference: LlamaForCausalLM + inject_ultimate_layers + flash_all_reduce"}
    res = {
        "metric": "tp_prefill_throughput_llama2_7b", "value": B * S / (ms / 1000.0), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "ttft_ms": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic: uniform random token ids, random-init N(0,0.02) weights",
        "config": {"model": cfg.name, "global_batch": B, "seq_len": S, "parallelism": f"tp{world} (MLP only)",
                   "allreduce": f"reference flash_all_reduce INT{args.bits} g{args.group_size} {args.quant_type}"},
        "clocks": clocks, "e2e": e2e, "impl": "reference",
    }
    return rank, res


def main():
    args = _parse()
    try:
        rank, res = run_reference(args) if args.impl == "reference" else run_ours(args)
    except SystemExit:
        raise
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            from quantized_flash_communication_b200.communication import reset_communicators
            reset_communicators()
            dist.destroy_process_group()
    except Exception:
        pass


if __name__ == "__main__":
    main()
