"""bfloat16 <-> float32 in numpy, bit-exact with torch's conversions (test infrastructure only).

bfloat16 is the top 16 bits of an IEEE float32. float32 -> bfloat16 rounds to nearest, ties to even, as
``torch.Tensor.to(torch.bfloat16)`` / ``type_as`` do (the cast at the end of the reference's ``apply_rope``,
omniasr_trt/modeling.py:306); NaN stays a quiet NaN.
"""

from __future__ import annotations

import numpy as np


def to_float32(bits: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def from_float32(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bfloat16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rounded = (u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | np.uint32(0x0040)).astype(np.uint16)
    return out


def round_trip(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (as float32)."""
    return to_float32(from_float32(x))
