"""Deterministic, platform-independent pseudo-random inputs for golden fixtures.

Values come from splitmix64 over a counter and are shaped with additions and
multiplications only (no transcendental functions), so every machine regenerates the same
bits.  `normal` is an Irwin-Hall approximation (sum of four uniforms, rescaled to unit
variance), which is all the fixtures need.
"""

from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix64(counter: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = counter + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def uniform(seed: int, count: int, stream: int = 0) -> np.ndarray:
    """float64 uniforms in [0, 1) with 53 random bits."""
    base = np.uint64((seed * 0x10001 + stream) & 0xFFFFFFFF) << np.uint64(32)
    counter = base + np.arange(count, dtype=np.uint64) * np.uint64(4) + np.uint64(stream)
    return (_splitmix64(counter) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def normal(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    """float32 approximately N(0, scale^2) of the given shape."""
    count = int(np.prod(shape))
    total = uniform(seed, count, 0) + uniform(seed, count, 1) + uniform(seed, count, 2) + uniform(seed, count, 3)
    values = (total - 2.0) * 1.7320508075688772 * scale
    return values.astype(np.float32).reshape(shape)


def integers(seed: int, count: int, high: int) -> np.ndarray:
    """int64 values in [0, high)."""
    return (uniform(seed, count, 7) * high).astype(np.int64)


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round float32 values to bf16 (nearest even) and return the raw uint16 bits."""
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def bf16_values(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)
