"""The C++ host mirror (darknet_zig_b200/host/gpu.hpp) and its gputest program
(tests/cpp/gputest.cpp): it builds against libdnb200.so on the CPU and lists its checks;
on a B200 every check must pass."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "cpp"))


@pytest.fixture(scope="module")
def gputest(built_lib, oracle):
    import build as cpp_build  # tests/cpp/build.py

    return cpp_build.build()


def test_cpp_mirror_builds_and_lists_its_checks(gputest):
    r = subprocess.run([gputest, "--list"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["elementwise", "biasAndNorm", "softmaxAndLoss", "pooling", "shortcutOp",
                                "fusedEntries"]


@pytest.mark.gpu
def test_cpp_gputest_passes_on_the_gpu(cuda, gputest):
    r = subprocess.run([gputest], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "checks passed" in r.stdout
