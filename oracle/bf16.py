"""bfloat16 helpers for the oracle (test infrastructure).

numpy has no bfloat16, so bf16 tensors are carried as uint16 bit patterns.  Conversions follow the
IEEE rule torch uses for float32 -> bfloat16: round to nearest, ties to even, NaN kept quiet.
"""

import numpy as np


def to_f32(u16: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    u16 = np.ascontiguousarray(u16, dtype=np.uint16)
    return (u16.astype(np.uint32) << 16).view(np.float32)


def from_f32(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    nan = np.isnan(x)
    rounding = ((bits >> 16) & 1) + np.uint32(0x7FFF)
    out = ((bits + rounding) >> 16).astype(np.uint16)
    if nan.any():
        out = np.where(nan, ((bits >> 16) | 0x40).astype(np.uint16), out)
    return out


def round_f32(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32 (models a torch bf16 op result)."""
    return to_f32(from_f32(x))


def as_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Values of a tensor stored as `dtype` ("bf16" -> uint16 bits, "f32" -> float32) as float32."""
    if dtype == "bf16":
        return to_f32(x)
    return np.asarray(x, dtype=np.float32)


def store(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values -> storage of `dtype` (uint16 bits for bf16)."""
    if dtype == "bf16":
        return from_f32(x)
    return np.asarray(x, dtype=np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to `dtype` precision and return them as float32."""
    if dtype == "bf16":
        return round_f32(x)
    return np.asarray(x, dtype=np.float32)
