"""Clock sampler against a fake ``nvidia-smi`` on PATH (no GPU, no real query)."""
import os
import stat
import time

from oscar_b200.utils.clocks import ClockSampler

FAKE = """#!/bin/sh
sleep 0.3
while true; do
  echo "0, 1965, 1965, 700.5, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
  sleep 0.05
done
"""


def _install(tmp_path, monkeypatch):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")


def test_short_region_still_gets_a_sample(tmp_path, monkeypatch):
    _install(tmp_path, monkeypatch)
    s = ClockSampler(period_ms=50)
    with s:
        time.sleep(0.01)  # a region far shorter than the tool's start-up delay
    out = s.summary()
    assert out["samples"] >= 1
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]


def test_missing_tool_reports_no_samples(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    s = ClockSampler()
    with s:
        pass
    assert s.summary()["samples"] == 0
