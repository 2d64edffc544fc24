"""Seeded synthetic inputs (numpy, host) shared by the tests and bench.py.

splitmix64 over the element index gives a reproducible stream on any host;
uniform[-1, 1) is (u >> 11) * 2^-53 * 2 - 1, normals come from Box-Muller
in fp64, integers in [-127, 127] from u mod 255.  16-bit values are rounded
to nearest-even; the arrays hold their bit patterns as uint16.
"""
from __future__ import annotations

import numpy as np

_G = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + np.arange(1, n + 1, dtype=np.uint64) * _G
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, n: int) -> np.ndarray:
    """fp64 uniform in [-1, 1)."""
    u = (splitmix64(seed, n) >> np.uint64(11)).astype(np.float64)
    return u * (2.0 ** -52) - 1.0


def normal(seed: int, n: int) -> np.ndarray:
    """fp64 standard normals (Box-Muller)."""
    m = (n + 1) // 2
    u = (splitmix64(seed, 2 * m) >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
    u1 = np.maximum(u[:m], 2.0 ** -53)
    u2 = u[m:]
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * m)
    out[:m] = r * np.cos(2 * np.pi * u2)
    out[m:] = r * np.sin(2 * np.pi * u2)
    return out[:n]


def int8(seed: int, n: int) -> np.ndarray:
    """int8 uniform over [-127, 127]."""
    return ((splitmix64(seed, n) % np.uint64(255)).astype(np.int64) - 127).astype(np.int8)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))
    return (u >> np.uint64(16)).astype(np.uint16)


def to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def bits_to_float(bits: np.ndarray, kind: str) -> np.ndarray:
    if kind == "bf16":
        return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def make(kind: str, dist: str, seed: int, n: int, scale: float = 1.0) -> np.ndarray:
    """n values of `dist` ('normal', 'uniform', 'int8') times `scale`, as
    kind 'f32' (float32), 'f16'/'bf16' (uint16 bits) or 'i8' (int8)."""
    if dist == "int8" or kind == "i8":
        return int8(seed, n)
    x = (normal(seed, n) if dist == "normal" else uniform(seed, n)) * scale
    if kind == "f32":
        return x.astype(np.float32)
    if kind == "bf16":
        return to_bf16_bits(x.astype(np.float32))
    if kind == "f16":
        return to_f16_bits(x)
    raise ValueError(kind)
