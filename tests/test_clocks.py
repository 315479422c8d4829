"""Clock sampling around a timed region, against a fake nvidia-smi on PATH (prints CSV rows)."""
import os
import stat
import time

from tutti_b200.common.clocks import ClockSampler

FAKE = """#!/bin/sh
i=0
while [ $i -lt 200 ]; do
  echo "0, 1965, 1965, 700.5, Not Active, Not Active, Not Active, Not Active"
  echo "0, 1500, 1965, 990.1, Not Active, Not Active, Not Active, Active"
  echo "1, 900, 1965, 300.0, Active, Not Active, Not Active, Not Active"
  echo "[N/A], x"
  i=$((i+1))
  sleep 0.05
done
"""


def test_sampler_reports_median_max_and_active_reasons_of_its_gpus(tmp_path, monkeypatch):
    smi = tmp_path / "nvidia-smi"
    smi.write_text(FAKE)
    smi.chmod(smi.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    s = ClockSampler([0]).start()
    time.sleep(0.3)
    r = s.stop()
    assert r["samples"] >= 2 and r["sm_max_mhz"] == 1965.0
    assert 1500.0 <= r["sm_mhz"] <= 1965.0
    assert r["reasons"] == ["sw_power_cap"]  # GPU 1's hw_slowdown is not this job's


def test_sampler_without_nvidia_smi_says_unsampled(monkeypatch, tmp_path):
    monkeypatch.setenv("PATH", str(tmp_path))
    assert ClockSampler([0]).start().stop() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
