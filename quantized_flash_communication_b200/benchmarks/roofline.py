"""Lower bounds of the prefill step's operators, for per-operator roofline fractions.

``op_bounds`` gives, for every region the model times (the names ``models/llama.py``
passes to ``maybe_region``), the least time one call can take on one rank: the slower of
its FLOPs at the bf16 tensor peak and its HBM bytes at the copy bandwidth, and for the
regions that contain an all-reduce also the bytes this rank pushes over NVLink at the
measured peer bandwidth.  ``bench.py --breakdown`` divides these by the measured times.

FLOPs: 2 m n k per GEMM; causal attention 2 B h S^2 d (QK^T and PV, each over half the
square).  HBM bytes: the operands read once and the result written once (bf16).  NVLink
bytes per two-shot all-reduce of n elements: (W - 1) / W n (b1 + b2), b = bytes per
element of each phase (payload + fp16 scale and zero per group of ``gs``).
"""
from __future__ import annotations

from typing import Dict

LINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200s


def _per_elem(p: int, gs: int) -> float:
    return 2.0 if p == 16 else p / 8.0 + 4.0 / gs


def allreduce_link_bytes(n: int, world: int, bits: int, gs: int) -> float:
    """Bytes one rank pushes over NVLink in a two-shot all-reduce of n elements."""
    if world <= 1:
        return 0.0
    from ..quantization import phase_bits
    p1, p2 = phase_bits(bits)
    return (world - 1) / world * n * (_per_elem(p1, gs) + _per_elem(p2, gs))


def op_bounds(cfg, B: int, S: int, world: int, bits: int, gs: int, peak_tflops: float, hbm_gbs: float,
              link_gbs: float = LINK_GBS) -> Dict[str, float]:
    """Region name -> lower bound in ms of one call on one rank."""
    M, H, hd = B * S, cfg.hidden_size, cfg.head_dim
    nq, nkv, inter = cfg.num_heads // world, cfg.num_kv_heads // world, cfg.intermediate_size // world

    def t_flops(f):
        return f / (peak_tflops * 1e12) * 1e3

    def t_hbm(b):
        return b / (hbm_gbs * 1e9) * 1e3

    def gemm(m, n, k, out_n=None):
        out_n = n if out_n is None else out_n
        return max(t_flops(2.0 * m * n * k), t_hbm(2.0 * (m * k + n * k + m * out_n)))

    t_link = allreduce_link_bytes(M * H, world, bits, gs) / (link_gbs * 1e9) * 1e3
    qkv_n = (nq + 2 * nkv) * hd
    qkv = gemm(M, qkv_n, H)
    rope = t_hbm(2.0 * (2 * M * (nq + nkv) * hd + 2 * M * nkv * hd))  # q, k read + written; k, v to the cache
    attn = max(t_flops(2.0 * B * nq * S * S * hd), t_hbm(2.0 * (M * qkv_n + M * nq * hd)))
    o_proj = gemm(M, H, nq * hd)
    gate_up = gemm(M, 2 * inter, H, out_n=inter)
    down = gemm(M, H, inter)
    norm = t_hbm(2.0 * 4 * M * H)  # x and residual in, residual and y out
    return {
        "qkv_gemm+rope_kv": qkv,
        "qkv_gemm": qkv,
        "rope_kv": rope,
        "attention": attn,
        "o_proj_gemm": o_proj,
        "o_proj_gemm+allreduce": max(o_proj, t_link),
        "o_proj_gemm+allreduce+norm": max(o_proj, t_link),
        "rmsnorm": norm,
        "gate_up_gemm_swiglu": gate_up,
        "down_gemm": down,
        "down_gemm+allreduce": max(down, t_link),
        "down_gemm+allreduce+norm": max(down, t_link),
        "  (allreduce part)": t_link,
        "  (allreduce+norm part)": t_link,
    }


def fractions(measured_ms_per_step: Dict[str, float], counts_per_step: Dict[str, int],
              bounds: Dict[str, float]) -> Dict[str, Dict[str, float]]:
    """Per region: the bound per step (bound per call x calls per step) and bound / measured.
    Regions without a bound (the GEMM part of a split region, whose shape differs between
    o_proj and down_proj) are left out."""
    out = {}
    for name, ms in measured_ms_per_step.items():
        if name not in bounds or ms <= 0:
            continue
        b = bounds[name] * counts_per_step.get(name, 0)
        out[name] = {"bound_ms_per_step": round(b, 4), "fraction": round(b / ms, 3)}
    return out
