"""Storage-type helpers for the oracle (TEST INFRASTRUCTURE ONLY, see ``oracle/__init__.py``).

numpy has no bfloat16, so bf16 tensors travel as their 16-bit patterns
(``int16`` / ``uint16``). The oracle keeps a bf16 pool in float32, which holds
every bf16 value exactly, and rounds results back with round-to-nearest-even.
"""

from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    u = np.asarray(bits).astype(np.uint16).astype(np.uint32) << np.uint32(16)
    return u.view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (nearest, ties to even); returns uint16 bit patterns. NaN stays NaN."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    out = rounded.astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    out[nan] = np.uint16(0x7FC0)
    return out


def to_compute(a: np.ndarray, dtype: str) -> np.ndarray:
    """Fixture array -> numpy array holding the exact stored values (bf16 as float32)."""
    if dtype == "bfloat16":
        return bf16_bits_to_f32(a)
    return np.asarray(a)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round exact results to the storage dtype, returned as float64 for comparisons."""
    if dtype == "bfloat16":
        return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, np.float32))).astype(np.float64)
    if dtype == "float16":
        return np.asarray(x).astype(np.float16).astype(np.float64)
    return np.asarray(x, np.float64)
