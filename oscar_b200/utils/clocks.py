"""Sample GPU SM clocks and throttle reasons with ``nvidia-smi`` while a region runs.

Read-only: it only queries clocks; it never changes any GPU setting.
"""
from __future__ import annotations

import os
import shutil
import statistics
import subprocess
import tempfile
import time

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """``nvidia-smi -lms`` in a child process for the duration of a ``with`` block.

    ``nvidia-smi`` takes a few hundred ms to print its first line, longer than a short timed
    region (5 decode steps at TP8 is ~100 ms), so ``__enter__`` waits until the first sample
    is written (at most ``first_sample_s``) before it returns.
    """

    def __init__(self, gpu_ids: list[str] | None = None, period_ms: int = 100, first_sample_s: float = 5.0):
        self.gpu_ids = gpu_ids
        self.period_ms = period_ms
        self.first_sample_s = first_sample_s
        self.proc = None
        self.out = None

    def __enter__(self):
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = [exe, f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"]
        if self.gpu_ids:
            cmd.append("-i=" + ",".join(self.gpu_ids))
        self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        deadline = time.monotonic() + self.first_sample_s
        while time.monotonic() < deadline and self.proc.poll() is None:
            if os.path.getsize(self.out.name) > 0:
                break
            time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.out is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi not found"}
        self.out.flush()
        with open(self.out.name) as f:
            lines = [ln.strip() for ln in f if ln.strip()]
        sm, mx, reasons, power = [], [], set(), []
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(REASONS, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        # median over samples under load (top half of the clock/power readings)
        loaded = sorted(sm)[len(sm) // 2:] if len(sm) > 4 else sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}
