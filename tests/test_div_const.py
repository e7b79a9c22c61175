"""The kernels' division by a per-launch constant (div_by_const in csrc/dnb_bn.cuh), restated
step for step with exact rational arithmetic for each fused multiply-add, must equal IEEE
float32 division t / d (round to nearest even) for every numerator it handles, at the
divisors the batchnorm backward meets (normalize_delta's element counts, blas.zig:200) and
a few awkward ones. On the GPU the same property is checked by every dx parity test whose
per-channel count is not a power of two."""
from __future__ import annotations

from fractions import Fraction

import numpy as np
import pytest

f32 = np.float32


def rn32(v: Fraction) -> np.float32:
    """The float32 nearest to v, ties to even."""
    f = f32(float(v))
    best = None
    for c in (np.nextafter(f, f32(-np.inf)), f, np.nextafter(f, f32(np.inf))):
        if not np.isfinite(c):
            continue
        key = (abs(Fraction(float(c)) - v), int(np.array(c).view(np.uint32)) & 1)
        if best is None or key < best[0]:
            best = (key, c)
    return best[1]


def fma(a, b, c) -> np.float32:
    return rn32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def div_by_const(t: np.float32, d: np.float32, r: np.float32) -> np.float32:
    at = abs(t)
    if not (at >= f32(2.0**-80) and at <= f32(2.0**96)):
        return f32(t / d)
    q0 = f32(t * r)
    q1 = fma(fma(-q0, d, t), r, q0)
    r1 = fma(-q1, d, t)
    step = 1 if (r1 > 0) == (q1 > 0) else -1
    q2 = np.array(np.array(q1, f32).view(np.int32) + step, np.int32).view(f32)[()]
    r2 = fma(-q2, d, t)
    return q2 if abs(r2) < abs(r1) else q1


DIVISORS = [3, 7, 140, 212, 1000, 3136, 6272, 100352, 200704, 401408, 802816, 1605632, 12345678, 6422528]


@pytest.mark.parametrize("d", DIVISORS)
def test_matches_ieee_division(d):
    rng = np.random.default_rng(d)
    n = 2500
    # typical normalize_delta terms, and magnitudes spread over the handled range and its edges
    t = np.concatenate([
        (rng.standard_normal(n // 2) * 1e-3).astype(f32),
        (rng.choice([-1, 1], n // 2) * 2.0 ** rng.uniform(-82, 98, n // 2)).astype(f32),
        np.array([0.0, -0.0, 1.0, -1.0, float(d), -float(d), 2.0**-80, 2.0**96, 2.0**-81, 3 * 2.0**96], f32),
    ])
    dd = f32(d)
    r = f32(f32(1) / dd)
    for v in t:
        got = div_by_const(v, dd, r)
        want = f32(v / dd)
        assert np.array(got, f32).view(np.uint32) == np.array(want, f32).view(np.uint32), (d, v, got, want)
