"""Seeded synthetic inputs for the parity tests, the golden fixtures and the benchmark.

The reference draws its test data from Zig's std.Random.DefaultPrng (src/utils.zig:11-57),
which cannot be replayed without a Zig toolchain. This module is this project's own
documented generator instead: splitmix64 over a counter, uniform floats from the top 24
bits, normals by Box-Muller in float64 rounded once to float32. It uses only integer
arithmetic and float64 math, so the bytes it produces do not depend on the numpy version
(unlike numpy's Generator methods, whose streams may change between releases).
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """n outputs of splitmix64 started at state seed + stream * 2**40 (uint64)."""
    with np.errstate(over="ignore"):
        base = np.uint64((int(seed) + (int(stream) << 40)) & 0xFFFFFFFFFFFFFFFF)
        z = base + (np.arange(1, n + 1, dtype=np.uint64) * _GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, shape, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    """float32 uniform on [lo, hi)."""
    n = int(np.prod(shape))
    u = (splitmix64(seed, n) >> np.uint64(40)).astype(np.float64) * (1.0 / 16777216.0)
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def normal(seed: int, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """float32 normal(mean, std) by Box-Muller."""
    n = int(np.prod(shape))
    u1 = ((splitmix64(seed, n, 1) >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)
    u2 = (splitmix64(seed, n, 2) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (mean + std * z).astype(np.float32).reshape(shape)


def class_ids(seed: int, batch: int, classes: int) -> np.ndarray:
    """Uniform class index per row (int64)."""
    return (splitmix64(seed, batch, 3) % np.uint64(classes)).astype(np.int64)


def one_hot(seed: int, batch: int, classes: int) -> np.ndarray:
    """Row-major [batch, classes] float32 one-hot truth at uniform class ids."""
    t = np.zeros((batch, classes), np.float32)
    t[np.arange(batch), class_ids(seed, batch, classes)] = 1.0
    return t
