"""The CPU oracle against the reference's own known-answer tests (CPU only).

Each test restates one `test` block of the reference and runs it against the C
restatement, pinning the oracle before anything is compared with it."""
from __future__ import annotations

import numpy as np
import pytest

from darknet_zig_b200 import synth

LEAKY, LOGISTIC, RELU, LINEAR = 7, 0, 1, 3


def test_leaky_kat(oracle):
    # activations.zig:145-150
    assert abs(oracle.activate(2.0, LEAKY) - 2.0) <= 1e-6
    assert abs(oracle.activate(-2.0, LEAKY) - (-0.2)) <= 1e-6
    assert abs(oracle.gradient(2.0, LEAKY) - 1.0) <= 1e-6
    assert abs(oracle.gradient(-0.2, LEAKY) - 0.1) <= 1e-6


def test_softmax_kat(oracle):
    # blas.zig:324-332
    x = np.array([1, 2, 3, 4], np.float32)
    out = np.zeros(4, np.float32)
    oracle.softmax(x, 4, 1, 4, 1, 4, 1, 1.0, out)
    assert abs(float(out.astype(np.float64).sum()) - 1.0) <= 1e-6
    assert out[3] > out[0]


def test_mean_variance_normalize_kat(oracle):
    # blas.zig:334-346: mean of [1..8] as batch 1 x 2 filters x 4 spatial
    x = np.arange(1, 9, dtype=np.float32)
    m = np.zeros(2, np.float32)
    v = np.zeros(2, np.float32)
    oracle.mean(x, 1, 2, 4, m)
    assert abs(m[0] - 2.5) <= 1e-6 and abs(m[1] - 6.5) <= 1e-6
    oracle.variance(x, m, 1, 2, 4, v)
    oracle.normalize(x, m, v, 1, 2, 4)
    s = 0.0
    for e in x[:4]:
        s = np.float32(s + e)
    assert abs(float(s)) <= 1e-5


def test_batchnorm_rolling_ema_closed_form(oracle):
    # smoke_test.zig:229-274: fixed input, 200 identical training steps, then
    # rolling = (1 - 0.99^200) * batch statistic (rel 1e-3), fraction in (0.86, 0.88)
    batch, w, h, c = 4, 3, 3, 2
    spatial = w * h
    x = synth.uniform(31, (batch * c * spatial,), -2.0, 2.0)
    y = np.zeros_like(x)
    scales = np.ones(c, np.float32)
    biases = np.zeros(c, np.float32)
    mean = np.zeros(c, np.float32)
    var = np.zeros(c, np.float32)
    rm = np.zeros(c, np.float32)
    rv = np.zeros(c, np.float32)
    steps = 200
    for _ in range(steps):
        oracle.bn_forward_layer(x, y, None, None, batch, c, spatial, scales, biases, mean, var, rm, rv, True, LINEAR)
    frac = 1.0 - np.float32(0.99) ** steps
    for i in range(c):
        assert abs(rm[i] - mean[i] * frac) <= 1e-3 * abs(mean[i] * frac)
        assert abs(rv[i] - var[i] * frac) <= 1e-3 * abs(var[i] * frac)
    assert 0.86 < frac < 0.88


def test_flat_index_decomposition_is_a_bijection():
    # smoke_test.zig:276-308: (b, j, i) from a flat id by % and / must cover every
    # element of [0, batch*n*size) once; the kernels decompose the same way
    batch, n, size = 3, 5, 7
    total = batch * n * size
    seen = np.zeros(total, np.int64)
    for flat in range(total):
        i = flat % size
        j = (flat // size) % n
        b = flat // (size * n)
        out = (b * n + j) * size + i
        assert out < total
        seen[out] += 1
    assert (seen == 1).all()


def _fastdiv_magic(d: int):
    """Restates FastDiv's constructor (csrc/dnb_common.cuh): l = ceil(log2 d),
    magic = floor(2^32 (2^l - d) / d) + 1, q = (t + ((n - t) >> 1)) >> (l - 1), t = mulhi."""
    l = 0
    while (1 << l) < d:
        l += 1
    magic = ((1 << 32) * ((1 << l) - d)) // d + 1
    return magic, l


@pytest.mark.parametrize("d", [1, 2, 3, 4, 5, 7, 49, 53, 196, 784, 1000, 1024, 3136, 12544, 50176, 65535, 131072,
                               (1 << 31) - 1, (1 << 31) + 11])
def test_fastdiv_restatement_exact(d):
    """The division by invariant integers the kernels use for index decomposition is
    exact for every 32-bit numerator (checked on edges and a random sample)."""
    magic, l = _fastdiv_magic(d)
    assert magic < (1 << 32)
    rng = np.random.default_rng(d)
    ns = np.concatenate([np.arange(0, 4096, dtype=np.uint64),
                         np.array([d - 1, d, d + 1, 2 * d - 1, 2 * d, (1 << 32) - 1, (1 << 32) - 2], np.uint64)
                         % np.uint64(1 << 32),
                         rng.integers(0, 1 << 32, 20000, dtype=np.uint64)])
    if d == 1:
        q = ns
    else:
        t = (ns * np.uint64(magic)) >> np.uint64(32)
        q = (t + ((ns - t) >> np.uint64(1))) >> np.uint64(l - 1)
    assert (q == ns // np.uint64(d)).all()
