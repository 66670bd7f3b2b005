"""Seeded synthetic tensors: SplitMix64 -> uniform [0, 1), Box-Muller -> N(0, 1).

One generator for inputs and weights, keyed by (base seed, tensor name), so the CUDA path, the CPU
oracle and the CPU baseline all see identical values without storing them.
"""
from __future__ import annotations

import numpy as np

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def name_seed(base: int, name: str) -> int:
    """FNV-1a of the tensor name mixed with the base seed."""
    h = 0xCBF29CE484222325 ^ (base & 0xFFFFFFFFFFFFFFFF)
    for ch in name.encode():
        h ^= ch
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def splitmix64(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (np.arange(1, n + 1, dtype=np.uint64) * _GAMMA)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, shape, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    u = (splitmix64(seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def normal(seed: int, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    n = int(np.prod(shape))
    m = (n + 1) // 2
    r = splitmix64(seed, 2 * m)
    u = (r >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    u1, u2 = 1.0 - u[0::2], u[1::2]
    rad = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * m)
    z[0::2] = rad * np.cos(2 * np.pi * u2)
    z[1::2] = rad * np.sin(2 * np.pi * u2)
    return (mean + std * z[:n]).astype(np.float32).reshape(shape)


def _i64(c: int) -> int:
    """A uint64 constant as the int64 with the same bits."""
    return c - (1 << 64) if c >= 1 << 63 else c


def _splitmix64_torch(seed: int, start: int, n: int, device):
    """SplitMix64 outputs start+1 .. start+n as int64 tensors holding the uint64 bits (two's-complement
    products and masked shifts give the same bits as the uint64 arithmetic of splitmix64)."""
    import torch
    i = torch.arange(start + 1, start + n + 1, dtype=torch.int64, device=device)
    z = i * _i64(0x9E3779B97F4A7C15) + _i64(seed & 0xFFFFFFFFFFFFFFFF)
    z = (z ^ ((z >> 30) & ((1 << 34) - 1))) * _i64(0xBF58476D1CE4E5B9)
    z = (z ^ ((z >> 27) & ((1 << 37) - 1))) * _i64(0x94D049BB133111EB)
    return z ^ ((z >> 31) & ((1 << 33) - 1))


def uniform_torch(seed: int, shape, device, lo: float = 0.0, hi: float = 1.0, chunk: int = 1 << 26):
    """uniform() computed with torch on `device` (bit-identical values; seconds instead of minutes for
    the det N=256 input). Generated in chunks of `chunk` elements to bound the int64 temporaries."""
    import torch
    n = int(np.prod(shape))
    out = torch.empty(n, dtype=torch.float32, device=device)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        z = _splitmix64_torch(seed, s, m, device)
        u = ((z >> 11) & ((1 << 53) - 1)).to(torch.float64) * (1.0 / 9007199254740992.0)
        out[s:s + m] = (lo + (hi - lo) * u).to(torch.float32)
    return out.reshape(shape)


def bytes_torch(seed: int, shape, device, chunk: int = 1 << 26):
    """Rng.bytes() computed with torch on `device` (bit-identical)."""
    import torch
    n = int(np.prod(shape))
    out = torch.empty(n, dtype=torch.uint8, device=device)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        z = _splitmix64_torch(seed, s, m, device)
        out[s:s + m] = ((z >> 56) & 0xFF).to(torch.uint8)
    return out.reshape(shape)


class Rng:
    """Named-tensor generator: Rng(seed).normal('conv1.w', shape, std)."""

    def __init__(self, seed: int = 2024):
        self.seed = seed

    def uniform(self, name: str, shape, lo=0.0, hi=1.0):
        return uniform(name_seed(self.seed, name), shape, lo, hi)

    def bytes(self, name: str, shape) -> np.ndarray:
        """Seeded uniform u8 values (synthetic image pixels)."""
        return (splitmix64(name_seed(self.seed, name), int(np.prod(shape))) >> np.uint64(56)).astype(np.uint8).reshape(shape)

    def normal(self, name: str, shape, std=1.0, mean=0.0):
        return normal(name_seed(self.seed, name), shape, std, mean)

    def uniform_torch(self, name: str, shape, device, lo=0.0, hi=1.0):
        return uniform_torch(name_seed(self.seed, name), shape, device, lo, hi)

    def bytes_torch(self, name: str, shape, device):
        return bytes_torch(name_seed(self.seed, name), shape, device)
