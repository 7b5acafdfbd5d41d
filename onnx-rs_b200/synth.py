"""Seeded synthetic inputs shared by the tests, the benchmark and the oracle.

Generator: SplitMix64 (Steele, Lea & Flood, 2014) over a counter, one stream per
(seed, tensor name).  uniform(): the top 24 bits -> [0, 1) exactly in fp32.
normal(): Box-Muller on pairs of 53-bit uniforms, computed in float64 and
rounded to fp32.  Everything is vectorised numpy, so a given (seed, name)
yields the same array on every machine.
"""
from __future__ import annotations

import zlib

import numpy as np

_G = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _stream_seed(seed: int, name: str) -> np.uint64:
    return np.uint64(((int(seed) & 0xFFFFFFFF) << 32) ^ zlib.crc32(name.encode()))


def splitmix64(seed: np.uint64, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = seed + (np.arange(1, n + 1, dtype=np.uint64) * _G)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, name: str, shape, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    u = (splitmix64(_stream_seed(seed, name), n) >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def normal(seed: int, name: str, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    m = (n + 1) // 2
    z = splitmix64(_stream_seed(seed, name), 2 * m)
    u = (z >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
    u1 = 1.0 - u[:m]  # (0, 1]
    u2 = u[m:]
    r = np.sqrt(-2.0 * np.log(u1))
    t = 2.0 * np.pi * u2
    out = np.empty(2 * m, np.float64)
    out[:m] = r * np.cos(t)
    out[m:] = r * np.sin(t)
    return (mean + std * out[:n]).astype(np.float32).reshape(shape)
