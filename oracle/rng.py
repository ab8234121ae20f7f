"""Seeded splitmix64 stream (numpy) — test infrastructure.

Fixtures regenerate their inputs from a seed with this generator, so the
committed golden files only need to hold the outputs; the stream does not
depend on numpy's Generator implementation or version.
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def u64(seed: int, n: int) -> np.ndarray:
    """n splitmix64 outputs for the given seed."""
    with np.errstate(over="ignore"):
        z = (np.uint64(seed) + _GOLD * np.arange(1, n + 1, dtype=np.uint64))
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def bytes_(seed: int, n: int) -> np.ndarray:
    words = u64(seed, (n + 7) // 8)
    return words.view(np.uint8)[:n].copy()


def uniform(seed: int, n: int) -> np.ndarray:
    """float64 in [0, 1) from the top 53 bits."""
    return (u64(seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))


def normal(seed: int, n: int) -> np.ndarray:
    """Standard normals by Box-Muller over two uniform streams (float64)."""
    u1 = uniform(seed, n)
    u2 = uniform(seed ^ 0x5DEECE66D, n)
    return np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)


def permutation(seed: int, n: int) -> np.ndarray:
    return np.argsort(u64(seed, n), kind="stable").astype(np.int32)
