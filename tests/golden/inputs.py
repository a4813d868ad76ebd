"""Deterministic test inputs, reproducible anywhere with numpy alone.

Uniform BF16 values in [lo, hi) from a SplitMix64 counter hash, the same
distribution the reference's kernel tests draw (testing/util/random.hpp:13-20
uses uniform(-2, 2) rounded to BF16), but with a generator whose stream is
fixed by this file rather than by a standard-library implementation.
"""
from __future__ import annotations

import numpy as np

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def _mix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def uniform_bf16(seed: int, shape, lo: float = -2.0, hi: float = 2.0) -> np.ndarray:
    """BF16 bits (uint16) of uniform values in [lo, hi)."""
    n = int(np.prod(shape))
    key = _mix64(np.array([seed], np.uint64))[0]
    h = _mix64(np.arange(n, dtype=np.uint64) ^ key)
    u = (h >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    v = (np.float32(lo) + np.float32(hi - lo) * u.astype(np.float32)).astype(np.float32)
    return f32_to_bf16(v).reshape(shape)


def uniform_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    key = _mix64(np.array([seed ^ 0xA5A5], np.uint64))[0]
    h = _mix64(np.arange(n, dtype=np.uint64) ^ key)
    return ((h >> np.uint64(32)) * np.uint64(vocab) >> np.uint64(32)).astype(np.uint32)
