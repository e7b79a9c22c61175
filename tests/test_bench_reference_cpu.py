"""bench.py's reference arm on the CPU: `--impl reference` times the reference's CPU op
sequence (the oracle restatement) and prints one JSON line with the keys the driver reads
(metric, value, unit, impl, cpu_baseline, e2e with zero copy bytes). Without a GPU the
reference's GPU kernels are left out of the line rather than failing it."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line(oracle):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3",
                        "--shape", "4,8,16,16", "--sgd-weights", "4096"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "config"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "gpu_kernels" not in d
