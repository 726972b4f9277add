"""Seeded Q4_K / Q6_K / Q8_0 super-block generators -- TEST INFRASTRUCTURE ONLY.

Value distributions follow the benchmark configurations of the reference path:
  Q4_K: fp16 d, dmin = |N(0,1)| * 1e-3; 12 packed scale bytes uniform (every
        byte pattern decodes to valid 6-bit (scale, min) pairs, and uniform
        bytes give uniform pairs in [0, 63]); 128 nibble bytes uniform.
  Q6_K: ql, qh bytes uniform; int8 sub-block scales uniform in [-32, 31];
        fp16 d = +-|N(0,1)| * 1e-3.
  Q8_0: fp16 d = |N(0,1)| * 1e-2; int8 quants uniform.
Block layouts: reference kernels.cu:3-13 (Q4_K, Q6_K) and kernels.cu:242-246 (Q8_0).
"""
from __future__ import annotations

import numpy as np

Q4K_BYTES, Q6K_BYTES, Q80_BYTES = 144, 210, 34


def _f16_bits(v: np.ndarray) -> np.ndarray:
    return np.asarray(v, dtype=np.float32).astype(np.float16).view(np.uint16)


def q4k_blocks(rng: np.random.Generator, n: int, mode: str = "baseline") -> np.ndarray:
    """n Q4_K blocks as uint8 [n, 144].

    mode: "baseline" (distributions above), "subnormal" (d and dmin forced
    subnormal), "zero_scale" (d = dmin = 0), "large" (d, dmin up to 60000),
    "mixed" (a mix of all of the above per block)."""
    b = rng.integers(0, 256, size=(n, Q4K_BYTES), dtype=np.uint8)
    d = np.abs(rng.standard_normal(n)) * 1e-3
    dm = np.abs(rng.standard_normal(n)) * 1e-3
    dbits, mbits = _f16_bits(d), _f16_bits(dm)
    if mode == "subnormal":
        dbits = rng.integers(1, 0x400, size=n, dtype=np.uint16)
        mbits = rng.integers(1, 0x400, size=n, dtype=np.uint16)
    elif mode == "zero_scale":
        dbits[:] = 0
        mbits[:] = 0
    elif mode == "large":
        dbits = _f16_bits(rng.uniform(1.0, 60000.0, n))
        mbits = _f16_bits(rng.uniform(1.0, 60000.0, n))
    elif mode == "mixed":
        k = rng.integers(0, 4, size=n)
        sub = rng.integers(1, 0x400, size=n, dtype=np.uint16)
        dbits = np.where(k == 1, sub, dbits)
        mbits = np.where(k == 2, sub, mbits)
        dbits = np.where(k == 3, 0, dbits).astype(np.uint16)
    b[:, 0:2] = dbits.astype("<u2").view(np.uint8).reshape(n, 2)
    b[:, 2:4] = mbits.astype("<u2").view(np.uint8).reshape(n, 2)
    return b


def q6k_blocks(rng: np.random.Generator, n: int, mode: str = "baseline") -> np.ndarray:
    """n Q6_K blocks as uint8 [n, 210]; modes as for q4k_blocks."""
    b = rng.integers(0, 256, size=(n, Q6K_BYTES), dtype=np.uint8)
    sc = rng.integers(-32, 32, size=(n, 16)).astype(np.int8)
    b[:, 192:208] = sc.view(np.uint8)
    sign = np.where(rng.integers(0, 2, size=n) == 1, -1.0, 1.0)
    dbits = _f16_bits(sign * np.abs(rng.standard_normal(n)) * 1e-3)
    if mode == "subnormal":
        dbits = rng.integers(1, 0x400, size=n, dtype=np.uint16) | np.where(sign < 0, 0x8000, 0).astype(np.uint16)
    elif mode == "zero_scale":
        dbits[:] = 0
    elif mode == "large":
        dbits = _f16_bits(sign * rng.uniform(1.0, 60000.0, n))
        b[:, 192:208] = rng.integers(-128, 128, size=(n, 16)).astype(np.int8).view(np.uint8)
    elif mode == "mixed":
        k = rng.integers(0, 3, size=n)
        sub = rng.integers(1, 0x400, size=n, dtype=np.uint16)
        dbits = np.where(k == 1, sub, dbits)
        dbits = np.where(k == 2, 0, dbits).astype(np.uint16)
        full = rng.integers(-128, 128, size=(n, 16)).astype(np.int8).view(np.uint8)
        b[:, 192:208] = np.where((k == 0)[:, None], full, b[:, 192:208])
    b[:, 208:210] = dbits.astype("<u2").view(np.uint8).reshape(n, 2)
    return b


def q8_0_blocks(rng: np.random.Generator, n: int) -> np.ndarray:
    b = rng.integers(0, 256, size=(n, Q80_BYTES), dtype=np.uint8)
    dbits = _f16_bits(np.abs(rng.standard_normal(n)) * 1e-2)
    b[:, 0:2] = dbits.astype("<u2").view(np.uint8).reshape(n, 2)
    return b


def kat_q4k_block() -> np.ndarray:
    """The reference's Q4_K known-answer block (dequant_q4k_cpu.c:181-217,
    kernels.cu:411-446): d = 1.0, dmin = 0, every (scale, min) = (1, 0),
    every quant byte 0x59.  Expected: elements 64g+0..31 = 9.0, 64g+32..63 = 5.0."""
    b = np.zeros(Q4K_BYTES, dtype=np.uint8)
    b[0:2] = np.array([0x00, 0x3C], dtype=np.uint8)
    b[4:8] = 1
    b[8:12] = 0
    b[12:16] = 1
    b[16:] = 0x59
    return b


def kat_q6k_block() -> np.ndarray:
    """The reference's Q6_K known-answer block (dequant_q4k_cpu.c:257-265):
    d = 1.0, every scale 1, ql = 0x88, qh = 0xAA.  Expected: all 256 = 8.0."""
    b = np.zeros(Q6K_BYTES, dtype=np.uint8)
    b[0:128] = 0x88
    b[128:192] = 0xAA
    b[192:208] = 1
    b[208:210] = np.array([0x00, 0x3C], dtype=np.uint8)
    return b


def matrix(qtype: int, rng: np.random.Generator, rows: int, cols: int, mode: str = "baseline") -> np.ndarray:
    """A [rows x cols] weight matrix in GGUF row-major block order, flat uint8."""
    if qtype == 12:
        return q4k_blocks(rng, rows * cols // 256, mode).reshape(-1)
    if qtype == 14:
        return q6k_blocks(rng, rows * cols // 256, mode).reshape(-1)
    if qtype == 8:
        return q8_0_blocks(rng, rows * cols // 32).reshape(-1)
    raise ValueError(qtype)
