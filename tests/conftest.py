"""Shared fixtures. Tests marked `gpu` need a CUDA device and the built libdnb200.so; they
fail (never skip) when either is missing, so a GPU run that silently falls back cannot
pass. Everything else runs on the CPU."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libdnb200.so")
    config.addinivalue_line("markers", "slow: full BASELINE-size case")


def pytest_terminal_summary(terminalreporter):
    """The plain |exact|-relative error of every reduction checked against the terms'
    2-norm bar (parity.py), worst case per check, beside the fraction of the bar it used."""
    try:
        from parity import PLAIN_REL
    except ImportError:
        return
    if not PLAIN_REL:
        return
    tr = terminalreporter
    tr.write_sep("-", "reductions: worst plain relative error |got-exact|/|exact| (and share of the bar used)")
    for name in sorted(PLAIN_REL):
        plain, of_bar = PLAIN_REL[name]
        tr.write_line(f"{name:40s} plain rel {plain:9.3g}   of bar {of_bar:6.3f}")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import get_oracle

    return get_oracle()


@pytest.fixture(scope="session")
def ref_emulation():
    from oracle.oracle import RefEmulation

    try:
        return RefEmulation()
    except FileNotFoundError as e:
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def built_lib():
    """Path of libdnb200.so, (re)building it first when a source is newer (nvcc
    cross-compiles, so this works without a GPU). On a box without nvcc the prebuilt
    library is used as is."""
    from darknet_zig_b200 import build

    if build.nvcc_path():
        build.build()
    assert os.path.exists(build.LIB), "libdnb200.so is missing and cannot be built here"
    return build.LIB


@pytest.fixture(scope="session")
def cuda(built_lib):
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    from darknet_zig_b200 import gpu

    gpu.init(0)
    return torch.device("cuda", 0)
