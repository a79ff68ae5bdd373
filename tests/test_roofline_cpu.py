"""Per-operator lower bounds of the prefill step (benchmarks/roofline.py)."""
import importlib.util
import os

import pytest

from quantized_flash_communication_b200.benchmarks.roofline import allreduce_link_bytes, fractions, op_bounds
from quantized_flash_communication_b200.models.config import get_config

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("world", [1, 2, 8])
def test_compute_bounds_add_up_to_the_step(world):
    """The compute-bound regions of every layer add up to the step's FLOPs (less the
    lm_head) at the same peak, split over the ranks."""
    cfg = get_config("llama2-7b")
    B, S, peak = 8, 1024, 1000.0
    b = op_bounds(cfg, B, S, world, 8, 128, peak, 1e9)  # HBM so fast that compute decides
    per_layer = b["qkv_gemm"] + b["attention"] + b["o_proj_gemm"] + b["gate_up_gemm_swiglu"] + b["down_gemm"]
    flops = _bench()._step_flops(cfg, B, S) - 2 * B * cfg.hidden_size * cfg.vocab_size
    assert per_layer * cfg.num_layers == pytest.approx(flops / world / (peak * 1e12) * 1e3, rel=1e-9)


def test_link_bytes_match_the_bench_formula():
    cfg = get_config("llama2-7b")
    wire = _bench()._wire_bytes_per_step(cfg, 8, 1024, 8, 8, 128)
    assert wire == pytest.approx(cfg.num_layers * 2 * allreduce_link_bytes(8 * 1024 * cfg.hidden_size, 8, 8, 128))
    assert allreduce_link_bytes(1000, 1, 8, 128) == 0.0


def test_fractions_skip_unbounded_regions():
    fr = fractions({"attention": 2.0, "  (gemm part)": 1.0}, {"attention": 32, "  (gemm part)": 64},
                   {"attention": 0.05})
    assert fr == {"attention": {"bound_ms_per_step": 1.6, "fraction": 0.8}}


def test_allreduce_sweep_uses_the_same_link_bytes():
    """bench_allreduce's roofline and the step's share one formula for the two-shot."""
    from quantized_flash_communication_b200.benchmarks.bench_allreduce import _wire_bytes
    for n, W, bits, gs in [(4096 * 16384, 8, 8, 128), (4096 * 1024, 4, 4, 32), (8192 * 4096, 2, 6, 64)]:
        assert _wire_bytes(n, W, bits, gs, False) == pytest.approx(allreduce_link_bytes(n, W, bits, gs))
    # one-shot: every rank pushes its whole quantized tensor to each of the W - 1 peers
    assert _wire_bytes(4096, 8, 8, 128, True) == pytest.approx(7 * 4096 * (1 + 4 / 128))
