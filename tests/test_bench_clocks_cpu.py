"""The bench's clock record: the sampler process is started and ended by its own handle, every
line it printed during the timed region is a sample, and the throttle reasons come from the
per-reason fields (a fake nvidia-smi on the PATH stands in for the driver's tool)."""
from __future__ import annotations

import os
import stat
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

FAKE = """#!/bin/sh
# prints one sample per 10 ms, like `nvidia-smi --query-gpu=... -lms 10`
i=0
while true; do
  if [ $((i % 2)) -eq 0 ]; then r="Not Active"; else r="Active"; fi
  echo "1965, 1965, Not Active, Not Active, Not Active, $r"
  i=$((i + 1))
  sleep 0.01
done
"""


def test_sampler_parses_samples_and_reasons(tmp_path, monkeypatch):
    tool = tmp_path / "nvidia-smi"
    tool.write_text(FAKE)
    tool.chmod(tool.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    import bench

    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.2)
    rec = s.stop()
    assert rec["source"].startswith("nvidia-smi")
    assert rec["samples"] >= 5
    assert rec["sm_mhz"] == 1965.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"]
    assert s.proc.poll() is not None  # the sampler process has ended


def test_sampler_without_tool_falls_back(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))  # no nvidia-smi at all
    import bench

    s = bench.ClockSampler(0)
    s.start()
    rec = s.stop()
    assert rec is None or rec["samples"] == 1
