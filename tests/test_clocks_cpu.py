"""The clock sampler's summary (utils/clocks.py) on canned nvidia-smi output: the median
SM clock and the throttle reasons of the loaded samples, the GPU filter, malformed lines."""
import os
import tempfile

from quantized_flash_communication_b200.utils.clocks import ClockSampler

ROWS = [
    # index, sm, max, power, active mask, hw_slowdown, hw_thermal, sw_thermal, sw_power_cap
    "0, 1965, 1965, 120.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",  # idle
    "0, 1350, 1965, 990.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
    "0, 1400, 1965, 950.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
    "0, 1500, 1965, 700.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
    "1, 900, 1965, 800.0, 0x0000000000000008, Not Active, Not Active, Active, Not Active",
    "garbage line",
    "0, [N/A], 1965, 800.0, 0x0, Not Active, Not Active, Not Active, Not Active",
]


def _sampler(gpus=None):
    s = ClockSampler(gpus)
    fd, s.path = tempfile.mkstemp(suffix=".csv")
    with os.fdopen(fd, "w") as f:
        f.write("\n".join(ROWS) + "\n")
    return s


def test_loaded_samples_median_and_reasons():
    out = _sampler([0]).summary()
    assert out["samples"] == 3                     # the idle row (<= 200 W) is left out
    assert out["sm_mhz"] == 1400.0                 # median of 1350, 1400, 1500
    assert out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    assert out["power_w_max"] == 990.1


def test_gpu_filter_keeps_other_gpus_reasons_apart():
    out = _sampler([1]).summary()
    assert out["samples"] == 1 and out["sm_mhz"] == 900.0
    assert out["reasons"] == ["sw_thermal_slowdown"]
    both = _sampler(None).summary()
    assert set(both["reasons"]) == {"sw_power_cap", "sw_thermal_slowdown"}


def test_without_nvidia_smi_the_summary_says_so():
    s = ClockSampler()
    assert s.summary()["reasons"] == ["nvidia-smi unavailable"]
