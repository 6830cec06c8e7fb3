"""bench.py's clock sampler (the contract's `clocks` key), driven by a fake nvidia-smi on PATH: it waits for the first
sample before the timed region, keeps only samples taken from then on (so a short region, as an 8-GPU run's ~0.15 s,
is still sampled), and reports the median SM clock under load and the active throttle reasons."""
import os
import stat
import time

import bench

FAKE = """#!/bin/sh
i=0
while true; do
  if [ $i -lt 3 ]; then echo "0, 345, 1965, 120.0, 0x1, Not Active, Not Active, Not Active, Not Active";
  else echo "0, 1800, 1965, 990.5, 0x4, Not Active, Not Active, Not Active, Active"; fi
  i=$((i+1)); sleep 0.05
done
"""


def test_sampler_keeps_samples_of_the_region_and_reasons(tmp_path, monkeypatch):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", str(tmp_path) + os.pathsep + os.environ["PATH"])
    with bench.ClockSampler(0) as clk:
        time.sleep(0.4)
    s = clk.summary()
    assert s["samples"] >= 2
    assert s["sm_mhz"] == 1800.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_sampler_without_nvidia_smi_reports_unsampled(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    with bench.ClockSampler(0) as clk:
        pass
    assert clk.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
