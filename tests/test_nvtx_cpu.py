"""Host-side switches of the native extension.  NVTX ranges: the switch reaches the
extension, wrapped ops keep their signatures (keywords, defaults, in-place outputs) and
an op's error still propagates.  The warps-per-row switch of the sequence-parallel kernel
and the stage switch of the two-shot kernel."""
import pytest
import torch

from quantized_flash_communication_b200._ext import _load
from quantized_flash_communication_b200.utils import trace

C = _load()
pytestmark = pytest.mark.skipif(C is None, reason="native extension not built")


def test_switch_reaches_extension():
    was = trace.nvtx_enabled()
    try:
        trace.set_nvtx(True)
        assert C.nvtx_enabled() and trace.nvtx_enabled()
        trace.set_nvtx(False)
        assert not C.nvtx_enabled() and not trace.nvtx_enabled()
    finally:
        trace.set_nvtx(was)


@pytest.mark.parametrize("on", [False, True])
def test_wrapped_op_keeps_signature_and_errors(on):
    was = trace.nvtx_enabled()
    try:
        trace.set_nvtx(on)
        x = torch.randn(4, 128)
        # keyword arguments and defaults are those of the unwrapped op
        with pytest.raises(RuntimeError):  # CPU tensor: the CUDA op refuses it
            C.argmax(logits=x, best_val=torch.empty(4), best_idx=torch.empty(4, dtype=torch.int64))
        with pytest.raises(TypeError):  # unknown keyword: pybind11 rejects it before the call
            C.gemm_bf16(x, x, nonexistent=1)
    finally:
        trace.set_nvtx(was)


def test_python_regions_nest_with_timer_absent():
    was = trace.nvtx_enabled()
    try:
        trace.set_nvtx(True)
        with trace.maybe_region(None, "outer"):
            with trace.maybe_region(None, "inner"):
                y = torch.ones(3) * 2
        assert torch.equal(y, torch.full((3,), 2.0))
        trace.set_nvtx(False)
        assert isinstance(trace.maybe_region(None, "x"), type(trace.contextlib.nullcontext()))
    finally:
        trace.set_nvtx(was)


def test_norm_warps_per_row_switch():
    """The sequence-parallel kernel's warps-per-row switch: values 1, 2, 4, 8, others refused."""
    from quantized_flash_communication_b200.parallel.quant_allreduce import set_norm_warps_per_row
    prev = set_norm_warps_per_row(4)
    try:
        assert set_norm_warps_per_row(2) == 4
        with pytest.raises(RuntimeError):
            set_norm_warps_per_row(3)
        assert set_norm_warps_per_row(2) == 2
    finally:
        set_norm_warps_per_row(prev)


def test_two_shot_stages_switch():
    from quantized_flash_communication_b200.parallel.quant_allreduce import set_two_shot_stages
    prev = set_two_shot_stages(2)
    try:
        assert set_two_shot_stages(1) == 2
        with pytest.raises(RuntimeError):
            set_two_shot_stages(3)
    finally:
        set_two_shot_stages(prev)


def test_gemv_switch():
    C.set_gemv(True)
    assert C.set_gemv(False) is True
