"""Seeded synthetic weights and activations in the reference's block layouts.

Distributions are the ones BASELINE.json's configs name (Q8_0: codes
U{-127..127}, scale U[0.001,0.02] rounded to f16 and stored as f32; Q4_K:
uniform nibbles and 6-bit scales/mins, d/dmin f16 U[1e-4,1e-3]; Q6_K: uniform
6-bit codes, i8 scales U{-127..127}, d f16 U[1e-5,1e-4]; x ~ N(0,1)).  Seeds
are derived per (config, tensor name) so every consumer sees identical bytes.
"""
from __future__ import annotations

import zlib

import numpy as np

from .formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0, row_bytes


def seed_of(*parts) -> int:
    """SplitMix64 of a CRC of the parts: a stable 64-bit seed per name."""
    z = (zlib.crc32("/".join(str(p) for p in parts).encode()) + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31)


def rng(*parts) -> np.random.Generator:
    return np.random.default_rng(seed_of(*parts))


def _f16_bits(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint16)


def random_weights(dtype: int, rows: int, cols: int, g: np.random.Generator) -> np.ndarray:
    """rows x cols matrix of random blocks, flat uint8 (row-major, reference layout)."""
    rb = row_bytes(dtype, cols)
    if rb is None:
        raise ValueError(f"cols={cols} is not a whole number of blocks for dtype {dtype}")
    if dtype == DTYPE_Q4_K:
        nb = rows * cols // 256
        blk = g.integers(0, 256, size=(nb, 144), dtype=np.uint8)
        blk[:, 0:2] = _f16_bits(g.uniform(1e-4, 1e-3, nb)).view(np.uint8).reshape(nb, 2)
        blk[:, 2:4] = _f16_bits(g.uniform(1e-4, 1e-3, nb)).view(np.uint8).reshape(nb, 2)
        return blk.reshape(-1)
    if dtype == DTYPE_Q6_K:
        nb = rows * cols // 256
        blk = g.integers(0, 256, size=(nb, 210), dtype=np.uint8)
        blk[:, 192:208] = g.integers(-127, 128, size=(nb, 16), dtype=np.int8).view(np.uint8)
        blk[:, 208:210] = _f16_bits(g.uniform(1e-5, 1e-4, nb)).view(np.uint8).reshape(nb, 2)
        return blk.reshape(-1)
    if dtype == DTYPE_Q8_0:
        nb = rows * cols // 32
        blk = np.empty((nb, 36), dtype=np.uint8)
        sc = g.uniform(0.001, 0.02, nb).astype(np.float16).astype(np.float32)
        blk[:, 0:4] = sc.view(np.uint8).reshape(nb, 4)
        blk[:, 4:] = g.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
        return blk.reshape(-1)
    raise ValueError(f"unsupported dtype {dtype}")


def randn(n: int, g: np.random.Generator) -> np.ndarray:
    return g.standard_normal(n, dtype=np.float32)


class Lcg:
    """The reference tests' LCG `azar` (crates/soso-llm-api/tests/cuda_matvec.rs:10-15)."""

    def __init__(self, state: int):
        self.s = state & 0xFFFFFFFFFFFFFFFF

    def next(self) -> int:
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return self.s >> 33


def _q4k_pack_scales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """(nb, 8) 6-bit scales and mins -> (nb, 12) packed bytes (the inverse of dequant.rs:150-167)."""
    q = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    q[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    q[:, 4:8] = (m[:, 0:4] & 63) | ((m[:, 4:8] >> 4) << 6)
    q[:, 8:12] = (sc[:, 4:8] & 15) | ((m[:, 4:8] & 15) << 4)
    return q


def model_weights(dtype: int, rows: int, cols: int, g: np.random.Generator, std: float | None = None) -> np.ndarray:
    """rows x cols blocks whose dequantised weights are zero-mean with standard deviation
    about `std` (default 1/sqrt(cols), like N(0, 1/cols) init), built directly in block
    form so a 3B-parameter model is generated in seconds.  Q4_K: uniform nibbles,
    scales U{32..63}, mins equal to the scales and dmin = 7.5 d, so every sub-block
    is centred; Q6_K: uniform 6-bit codes (q - 32 is centred), i8 scales of random sign
    and magnitude U{32..127}; Q8_0: uniform codes U{-127..127}."""
    s = (1.0 / np.sqrt(cols)) if std is None else std
    rb = row_bytes(dtype, cols)
    if rb is None:
        raise ValueError(f"cols={cols} is not a whole number of blocks for dtype {dtype}")
    if dtype == DTYPE_F32:  # (an f32 matrix, as the reference keeps its routers: N(0, s^2))
        return (g.standard_normal(rows * cols) * s).astype(np.float32).view(np.uint8)
    if dtype == DTYPE_Q4_K:
        nb = rows * cols // 256
        blk = np.empty((nb, 144), dtype=np.uint8)
        sc = g.integers(32, 64, size=(nb, 8), dtype=np.uint8)
        d = np.full(nb, s / (47.5 * 4.61), dtype=np.float32) * g.uniform(0.8, 1.25, nb).astype(np.float32)
        blk[:, 0:2] = _f16_bits(d).view(np.uint8).reshape(nb, 2)
        blk[:, 2:4] = _f16_bits(d * 7.5).view(np.uint8).reshape(nb, 2)
        blk[:, 4:16] = _q4k_pack_scales(sc, sc)
        blk[:, 16:] = g.integers(0, 256, size=(nb, 128), dtype=np.uint8)
        return blk.reshape(-1)
    if dtype == DTYPE_Q6_K:
        nb = rows * cols // 256
        blk = np.empty((nb, 210), dtype=np.uint8)
        blk[:, 0:192] = g.integers(0, 256, size=(nb, 192), dtype=np.uint8)
        mag = g.integers(32, 128, size=(nb, 16)).astype(np.int16)
        sgn = np.where(g.integers(0, 2, size=(nb, 16)) == 0, -1, 1).astype(np.int16)
        blk[:, 192:208] = (mag * sgn).astype(np.int8).view(np.uint8)
        d = np.full(nb, s / (18.5 * 80.0), dtype=np.float32) * g.uniform(0.8, 1.25, nb).astype(np.float32)
        blk[:, 208:210] = _f16_bits(d).view(np.uint8).reshape(nb, 2)
        return blk.reshape(-1)
    if dtype == DTYPE_Q8_0:
        nb = rows * cols // 32
        blk = np.empty((nb, 36), dtype=np.uint8)
        sc = (np.full(nb, s / 73.6, dtype=np.float32) * g.uniform(0.8, 1.25, nb).astype(np.float32))
        blk[:, 0:4] = sc.astype(np.float16).astype(np.float32).view(np.uint8).reshape(nb, 4)
        blk[:, 4:] = g.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
        return blk.reshape(-1)
    raise ValueError(f"unsupported dtype {dtype}")
