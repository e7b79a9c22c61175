"""Pins the C oracle against the reference's own kernel code (CPU only).

The reference's CPU path is Zig and cannot be built here; its device kernels are C++ and
can: oracle/build_oracle.py compiles src/kernels/darknet_kernels.hip for the host and
oracle/ref_emulate.cpp runs each kernel with the reference's launch shapes. The committed
fixtures (tests/golden/reference_gputest.{json,npz}, made by tests/golden/make_golden.py)
hold those outputs on the gputest cases, so this file runs without the reference tree;
when the emulation library is present the comparison is also made live.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import cases  # noqa: E402
from parity import assert_bitexact, assert_close, assert_value_equal  # noqa: E402

GOLDEN_JSON = os.path.join(HERE, "golden", "reference_gputest.json")
GOLDEN_NPZ = os.path.join(HERE, "golden", "reference_gputest.npz")


@pytest.fixture(scope="module")
def oracle_outputs(oracle):
    out, _ = cases.run_oracle(oracle, cases.inputs())
    return out


def _digest(a, value_class):
    a = np.ascontiguousarray(a)
    if value_class and a.dtype == np.float32:
        a = a + np.float32(0.0)
    return hashlib.sha256(a.tobytes()).hexdigest()


def test_golden_covers_every_output(oracle_outputs):
    digests = json.load(open(GOLDEN_JSON))
    arrays = np.load(GOLDEN_NPZ)
    assert set(digests) | set(arrays.files) == set(oracle_outputs)


def test_oracle_matches_reference_exact_digests(oracle_outputs):
    digests = json.load(open(GOLDEN_JSON))
    bad = [k for k, meta in digests.items()
           if _digest(oracle_outputs[k], meta["class"] == "value") != meta["sha256"]]
    assert not bad, f"oracle differs from the reference kernels on {bad}"


REDUCTIONS = {"backward_bias", "backward_scale", "mean", "variance", "mean_delta", "variance_delta"}


def _rtol(key):
    # reductions (212-term sums, tree vs sequential order) at the north_star bar; the
    # per-element ops differ by an ulp or two
    return 1e-5 if key in REDUCTIONS else 2e-6


def test_oracle_matches_reference_within_tolerance(oracle_outputs):
    arrays = np.load(GOLDEN_NPZ)
    for k in arrays.files:
        assert_close(oracle_outputs[k], arrays[k], name=k, rtol=_rtol(k), atol=1e-6)


def test_oracle_matches_live_reference_emulation(oracle, ref_emulation, oracle_outputs):
    d = cases.inputs()
    ref = cases.run_reference_all(ref_emulation, oracle, d)
    for k, want in ref.items():
        cls = cases.comparison_class(k)
        got = oracle_outputs[k]
        if cls == "exact":
            if got.dtype == np.float32:
                assert_bitexact(got, want, k)
            else:
                assert_value_equal(got, want, k)
        elif cls == "value":
            assert_value_equal(got, want, k)
        else:
            assert_close(got, want, name=k, rtol=_rtol(k), atol=1e-6)


def test_relu_sign_of_zero_is_the_cpu_one(oracle_outputs):
    """activations.zig:63 selects +0.0 for x <= 0; the reference kernel's x*(x>0) gives -0.0.
    The oracle (and the new kernels) follow the CPU code."""
    d = cases.inputs()
    neg = d["a"] < 0
    y = oracle_outputs["activate_1"]
    assert (np.signbit(y[neg]) == False).all()  # noqa: E712


def test_reference_gpu_bindings_match_the_launcher_signatures():
    """oracle/_ref/libref_gpu.so (the reference's kernels built for sm_100a) is bound with
    argtypes whose counts equal the C signatures in oracle/ref_gpu.cu, and a call with a
    wrong count is refused on the host (no device is touched)."""
    import re

    from oracle.oracle import RefGpu

    try:
        ref = RefGpu()
    except FileNotFoundError as e:
        pytest.skip(str(e))
    src = open(os.path.join(os.path.dirname(__file__), "..", "oracle", "ref_gpu.cu")).read()
    sigs = {m.group(1): m.group(2) for m in re.finditer(r"int ref_gpu_(\w+)\(([^)]*)\)", src)}
    for name in ("conv_bn_forward", "conv_bn_backward", "sgd_weights"):
        n_c = len([p for p in sigs[name].split(",") if p.strip()])
        assert len(getattr(ref.lib, "ref_gpu_" + name).argtypes) == n_c, name
    with pytest.raises(TypeError, match="takes 8 arguments"):
        ref._call("sgd_weights", 1, 0.1, 0.9, 5e-4, 1, 0, 0, 0, 0)
