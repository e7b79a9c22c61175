"""Builds tests/cpp/gputest (the C++ host mirror's CPU-vs-GPU comparison) with g++ against
libdnb200.so and the oracle's liboracle.so (test infrastructure), and tests/cpp/weights_rt
(a round trip through the C++ host's .weights code; host only).

    python tests/cpp/build.py      -> tests/cpp/_build/gputest, tests/cpp/_build/weights_rt
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "_build", "gputest")


def build() -> str:
    src = os.path.join(HERE, "gputest.cpp")
    hdr = os.path.join(ROOT, "darknet_zig_b200", "host", "gpu.hpp")
    lib = os.path.join(ROOT, "darknet_zig_b200", "libdnb200.so")
    orc = os.path.join(ROOT, "oracle", "_build", "liboracle.so")
    deps = [src, hdr, lib, orc, os.path.join(ROOT, "include", "dnb200.h")]
    if os.path.exists(OUT) and all(os.path.getmtime(OUT) >= os.path.getmtime(d) for d in deps if os.path.exists(d)):
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"), "-I",
           os.path.join(ROOT, "darknet_zig_b200", "host"), "-I", os.path.join(ROOT, "oracle"), src, "-o", OUT,
           "-L", os.path.dirname(lib), "-ldnb200", "-L", os.path.dirname(orc), "-loracle",
           "-Wl,-rpath,$ORIGIN/../../../darknet_zig_b200", "-Wl,-rpath,$ORIGIN/../../../oracle/_build"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed:\n{r.stdout}\n{r.stderr}")
    return OUT


WEIGHTS_RT = os.path.join(HERE, "_build", "weights_rt")


def build_weights_rt() -> str:
    src = os.path.join(HERE, "weights_rt.cpp")
    hdr = os.path.join(ROOT, "darknet_zig_b200", "host", "weights.hpp")
    if os.path.exists(WEIGHTS_RT) and all(os.path.getmtime(WEIGHTS_RT) >= os.path.getmtime(d) for d in (src, hdr)):
        return WEIGHTS_RT
    os.makedirs(os.path.dirname(WEIGHTS_RT), exist_ok=True)
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "darknet_zig_b200", "host"), src, "-o",
           WEIGHTS_RT]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed:\n{r.stdout}\n{r.stderr}")
    return WEIGHTS_RT


if __name__ == "__main__":
    print(build())
    print(build_weights_rt())
    sys.exit(0)
