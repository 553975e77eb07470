"""bf16 rounding on float32 numpy arrays (round to nearest, ties to even), NaN preserved.

Used by the oracle wherever the reference rounds a value to bf16 (`.to(tl.bfloat16)`, bf16 x bf16
products under Triton's promotion rules, torch `.to(torch.bfloat16)`).
"""

from __future__ import annotations

import numpy as np


def round_bf16(a) -> np.ndarray:
    """float32 values rounded to the nearest bf16 value (ties to even), returned as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    # finite values never overflow uint32 here (largest: 0xFF7FFFFF + 0x8000); NaNs are restored below
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    return np.where(np.isnan(a), a, out)


def bf16_bits_to_f32(bits) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def f32_to_bf16_bits(a) -> np.ndarray:
    """float32 -> uint16 bit patterns of the rounded bf16 values."""
    r = round_bf16(a)
    return (r.view(np.uint32) >> 16).astype(np.uint16)
