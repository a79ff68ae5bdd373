"""Sample GPU clocks and throttle reasons with nvidia-smi while a timed region runs.

Reads only (``--query-gpu``); never changes a clock or any other GPU setting.
"""
from __future__ import annotations

import csv
import io
import os
import shutil
import subprocess
import tempfile
from typing import Dict, List, Optional

_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_indices: Optional[List[int]] = None, period_ms: int = 200):
        self.gpus = gpu_indices
        self.period_ms = period_ms
        self.proc = None
        self.path = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="qfc_clocks_", suffix=".csv")
        os.close(fd)
        self._fh = open(self.path, "w")
        self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits",
                                      f"-lms={self.period_ms}"], stdout=self._fh, stderr=subprocess.DEVNULL)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._fh.close()
        return False

    def summary(self) -> Dict:
        if self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        rows = []
        with open(self.path) as f:
            for rec in csv.reader(io.StringIO(f.read())):
                if len(rec) < 9:
                    continue
                try:
                    idx = int(rec[0])
                    if self.gpus is not None and idx not in self.gpus:
                        continue
                    rows.append(dict(idx=idx, sm=float(rec[1]), smax=float(rec[2]), power=float(rec[3]),
                                     flags={r: rec[5 + i].strip() == "Active" for i, r in enumerate(_REASONS)}))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [r for r in rows if r["power"] > 200.0] or rows
        sms = sorted(r["sm"] for r in loaded)
        reasons = sorted({k for r in loaded for k, v in r["flags"].items() if v})
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": max(r["smax"] for r in rows), "reasons": reasons,
                "samples": len(loaded), "power_w_max": max(r["power"] for r in rows)}
