"""Float32 -> bfloat16 / float16 conversions (round to nearest, ties to even).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference has no bfloat16 type (namitorch/dtype.py:16-25); its float16 conversions
go through ``ndarray.astype(np.float16)`` (namitorch/tensor.py:541). bfloat16 here is the
upper 16 bits of the float32 pattern after adding the RNE bias, which is what an IEEE
round-to-nearest-even narrowing to an 8-bit-significand format computes. NaN inputs
map to the canonical quiet NaN 0x7FFF (the pattern the B200 conversion instruction
produces); comparisons treat any two NaNs as equal.
"""
from __future__ import annotations

import numpy as np

BF16_CANONICAL_NAN = np.uint16(0x7FFF)


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of RNE(float32 -> bfloat16)."""
    x = np.ascontiguousarray(values, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = BF16_CANONICAL_NAN
    return rounded


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bfloat16 bit patterns to float32."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_to_bf16(values: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (returned widened to float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(values))


def f32_to_f16_bits(values: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(values, dtype=np.float32).astype(np.float16).view(np.uint16)


def bits_equal_nan_aware(a_bits: np.ndarray, b_bits: np.ndarray, kind: str) -> bool:
    """Bit equality of two uint16 arrays where any NaN equals any NaN."""
    a = np.asarray(a_bits, dtype=np.uint16)
    b = np.asarray(b_bits, dtype=np.uint16)
    if a.shape != b.shape:
        return False
    if kind == "bf16":
        a_nan = ((a & 0x7F80) == 0x7F80) & ((a & 0x007F) != 0)
        b_nan = ((b & 0x7F80) == 0x7F80) & ((b & 0x007F) != 0)
    else:
        a_nan = ((a & 0x7C00) == 0x7C00) & ((a & 0x03FF) != 0)
        b_nan = ((b & 0x7C00) == 0x7C00) & ((b & 0x03FF) != 0)
    return bool(np.array_equal(a_nan, b_nan) and np.array_equal(a[~a_nan], b[~b_nan]))
