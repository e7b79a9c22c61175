"""Comparison helpers shared by the parity tests (not collected as tests).

Bars:
  * bit-exact (bit patterns equal; -0.0 and +0.0 differ) for fill/copy/scal/axpy/mul/
    add_scalar/constrain/shortcut, relu/leaky/linear and their gradients, bias/scale
    broadcasts, maxpool values and indices, and every per-element BN output given the
    per-channel statistics the kernel itself produced;
  * RTOL = 1e-5 relative / ATOL = 1e-6 absolute for reductions and transcendentals.
For a reduction the relative error is measured against max(|exact|, ||terms||_2): a sum of
many random-signed terms can cancel to near zero, where no fp32 summation (the
reference's own sequential one included) meets a bar relative to the tiny result. The
exact value is the same sum computed in float64 from the same float32 terms.
"""
from __future__ import annotations

import numpy as np

RTOL = 1e-5
ATOL = 1e-6


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bitexact(got, want, name=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, (name, got.shape, want.shape)
    bad = np.flatnonzero(bits(got).ravel() != bits(want).ravel())
    if bad.size:
        i = bad[0]
        raise AssertionError(f"{name}: {bad.size} of {got.size} elements differ in bits; first at {i}: "
                             f"got {got.ravel()[i]!r} want {want.ravel()[i]!r}")


def assert_value_equal(got, want, name=""):
    """Equal as floats (+0.0 == -0.0)."""
    got = np.asarray(got)
    want = np.asarray(want)
    bad = np.flatnonzero(got.ravel() != want.ravel())
    if bad.size:
        i = bad[0]
        raise AssertionError(f"{name}: {bad.size} elements differ; first at {i}: {got.ravel()[i]!r} vs "
                             f"{want.ravel()[i]!r}")


# Every reduction checked against the ||terms||_2 bar also records its plain relative error
# |got - exact| / |exact| here; conftest.py prints the worst per check at the end of the run,
# so the relaxation can be read next to the bar it replaces.
PLAIN_REL: dict[str, tuple[float, float]] = {}


def assert_close(got, want, name="", rtol=RTOL, atol=ATOL, scale=None):
    """|got - want| <= atol + rtol * max(|want|, scale)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    ref = np.abs(want) if scale is None else np.maximum(np.abs(want), np.asarray(scale, np.float64))
    err = np.abs(got - want)
    bound = atol + rtol * ref
    if scale is not None and err.size:
        key = name.split(" n=")[0]
        plain = float(np.max(err / np.maximum(np.abs(want), 1e-300)))
        of_bar = float(np.max(err / np.maximum(bound, 1e-300)))
        old = PLAIN_REL.get(key, (0.0, 0.0))
        PLAIN_REL[key] = (max(old[0], plain), max(old[1], of_bar))
    bad = np.flatnonzero((err > bound).ravel())
    if bad.size:
        i = bad[0]
        worst = int(np.argmax((err / np.maximum(bound, 1e-300)).ravel()))
        raise AssertionError(
            f"{name}: {bad.size} of {got.size} outside atol={atol} rtol={rtol}; first at {i}: got "
            f"{got.ravel()[i]!r} want {want.ravel()[i]!r}; worst at {worst}: got {got.ravel()[worst]!r} want "
            f"{want.ravel()[worst]!r}")


def channel_view(a: np.ndarray, batch: int, filters: int, spatial: int) -> np.ndarray:
    """[filters, batch*spatial] view of an NCHW tensor (a copy)."""
    return np.ascontiguousarray(a.reshape(batch, filters, spatial).transpose(1, 0, 2).reshape(filters, -1))


def exact_channel_sum(terms: np.ndarray, batch: int, filters: int, spatial: int):
    """float64 per-channel sum of float32 terms and the terms' per-channel 2-norm."""
    t = channel_view(terms, batch, filters, spatial).astype(np.float64)
    return t.sum(axis=1), np.sqrt((t * t).sum(axis=1))
