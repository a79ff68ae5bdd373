"""Standalone quantizer kernels against the reference's, on the same GPU.

    python -m quantized_flash_communication_b200.benchmarks.bench_quant [--n 67108864] [--reference]

For each op, one JSON line: device time (CUDA events, median of --iters, L2 flushed
between samples), the algorithmic bytes it must move, bandwidth and its fraction of the
measured copy bandwidth (MEASURED_PEAKS.json).  Ops, through the reference-compatible
entry points of both implementations (fp16 input, group 128, codes one per byte):

  quantize_int8_asym, quantize_int4_asym, quantize_int4_sym   kernels.triton_quantize
  dequantize                                                   kernels.triton_dequantize
  pack_int4, unpack_int4                                       kernels_jit.pack_int4 / unpack_int4

With --reference the unmodified reference's Triton quantizers (kernels.py:87-131) and its
JIT-compiled pack / unpack (kernels_jit.py:105-125) run on the same tensors; the line then
also carries the reference's time and the share of codes and scales on which the two agree.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

from .timing import median, time_fn


def _peak_hbm_gbs() -> float:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0  # the pool's earlier copy measurement


def _reference_modules():
    from .reference_arm import REF_DIR
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import kernels as ref_k  # noqa: E402  (reference, unmodified)
    import kernels_jit as ref_kj  # noqa: E402  (reference, unmodified; compiles its CUDA at import)
    return ref_k, ref_kj


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=1 << 26)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--reference", action="store_true")
    args = ap.parse_args(argv)
    from .. import kernels as K
    from .. import kernels_jit as KJ
    dev = torch.device("cuda", 0)
    n, gs = args.n, 128
    peak = _peak_hbm_gbs()
    g = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randn(n, generator=g).to(torch.float16).to(dev)
    ref_k = ref_kj = None
    if args.reference:
        ref_k, ref_kj = _reference_modules()
    meta = 4.0 * n / gs  # fp16 scale + fp16 zero per group

    q8, s8, z8 = K.triton_quantize(x, 8, gs, "asym")
    codes4 = torch.randint(0, 16, (n,), generator=g, dtype=torch.int8).to(dev)
    packed = KJ.pack_int4(codes4)
    ops = [
        ("quantize_int8_asym", 2.0 * n + n + meta, lambda m: m.triton_quantize(x, 8, gs, "asym")),
        ("quantize_int4_asym", 2.0 * n + n + meta, lambda m: m.triton_quantize(x, 4, gs, "asym")),
        ("quantize_int4_sym", 2.0 * n + n + meta, lambda m: m.triton_quantize(x, 4, gs, "sym")),
        ("dequantize", n + meta + 2.0 * n, lambda m: m.triton_dequantize(q8, s8, z8, x.shape, gs)),
        ("pack_int4", n + n / 2.0, lambda m: m.pack_int4(codes4)),
        ("unpack_int4", n / 2.0 + 2.0 * n, lambda m: m.unpack_int4(packed, codes4.shape)),
    ]
    for name, nbytes, call in ops:
        ours_mod = KJ if name in ("pack_int4", "unpack_int4") else K
        t = median(time_fn(lambda: call(ours_mod), iters=args.iters))
        rec = {"op": name, "n": n, "ms": t, "bytes": nbytes, "gbs": nbytes / (t * 1e-3) / 1e9,
               "fraction_of_measured_hbm": nbytes / (t * 1e-3) / 1e9 / peak}
        if ref_k is not None:
            ref_mod = ref_kj if name in ("pack_int4", "unpack_int4") else ref_k
            tr = median(time_fn(lambda: call(ref_mod), iters=args.iters))
            rec.update(reference_ms=tr, speedup_vs_reference=tr / t)
            a, b = call(ours_mod), call(ref_mod)
            if isinstance(a, tuple):  # (codes, scale, zero)
                rec["codes_equal_share"] = (a[0].view(torch.uint8) == b[0].view(torch.uint8)).float().mean().item()
                rec["scales_equal_share"] = (a[1] == b[1]).float().mean().item()
            else:
                rec["outputs_equal_share"] = (a.reshape(-1) == b.reshape(-1)).float().mean().item()
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
