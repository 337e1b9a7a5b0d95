"""Portable, bit-reproducible seeded inputs for parity tests (oracle side).

Values come from integer arithmetic only (splitmix64 counters), so the same
seed gives the same bytes on any machine, CPU type or numpy build:
  * ``normal``: Irwin-Hall sum of twelve 24-bit uniforms minus 6 (mean 0,
    variance 1, support [-6, 6]) as an exact float64, then rounded once to
    the requested 16-bit type (round to nearest even).
  * ``permutation``: argsort of splitmix64 keys.
16-bit types are returned as uint16 bit patterns (numpy has no bfloat16).
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(counter: np.ndarray) -> np.ndarray:
    """splitmix64 finaliser of ``counter + golden`` (wrapping uint64 arithmetic)."""
    with np.errstate(over="ignore"):
        z = counter.astype(np.uint64) + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _key(seed: int, stream: int) -> np.uint64:
    return splitmix64(np.array([seed * 1_000_003 + stream], dtype=np.uint64))[0]


def uniform_u64(seed: int, n: int, stream: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        ctr = np.arange(n, dtype=np.uint64) + _key(seed, stream)
    return splitmix64(ctr)


def normal_f64(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """n approximately standard-normal float64 values, exactly reproducible."""
    out = np.empty(n, dtype=np.float64)
    chunk = 1 << 20
    mask = np.uint64((1 << 24) - 1)
    for lo in range(0, n, chunk):
        m = min(chunk, n - lo)
        with np.errstate(over="ignore"):
            ctr = np.arange(lo * 6, (lo + m) * 6, dtype=np.uint64) + _key(seed, stream)
        r = splitmix64(ctr).reshape(m, 6)
        s = ((r & mask).astype(np.int64).sum(axis=1)
             + ((r >> np.uint64(32)) & mask).astype(np.int64).sum(axis=1))
        out[lo:lo + m] = (s - 6 * (1 << 24)) / float(1 << 24)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest even); returns uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        r = ((u + bias) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = np.uint16(0x7FC0)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


def to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    """uint16 bit patterns of `dtype` ('f16' | 'bf16') -> float32 (exact)."""
    if dtype == "bf16":
        return bf16_bits_to_f32(bits)
    if dtype == "f16":
        return f16_bits_to_f32(bits)
    raise ValueError(dtype)


def from_f64(x: np.ndarray, dtype: str) -> np.ndarray:
    """float64 -> uint16 bit patterns of `dtype`, one rounding (f16) or
    float64->float32->bf16 (both exact-then-RNE for Irwin-Hall values)."""
    if dtype == "f16":
        return np.asarray(x, dtype=np.float64).astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return f32_to_bf16_bits(np.asarray(x, dtype=np.float64).astype(np.float32))
    raise ValueError(dtype)


def normal(seed: int, shape: tuple[int, ...], dtype: str, stream: int = 0) -> np.ndarray:
    """Seeded N(0,1)-like values as uint16 bit patterns of `dtype`."""
    n = int(np.prod(shape)) if shape else 1
    return from_f64(normal_f64(seed, n, stream), dtype).reshape(shape)


def permutation(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """A seeded permutation of range(n) (int64)."""
    return np.argsort(uniform_u64(seed, n, stream), kind="stable").astype(np.int64)


def randint(seed: int, n: int, lo: int, hi: int, stream: int = 0) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive), int64."""
    span = np.uint64(hi - lo + 1)
    return (uniform_u64(seed, n, stream) % span).astype(np.int64) + lo
