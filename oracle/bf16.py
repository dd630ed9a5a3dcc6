"""bfloat16 emulation in numpy (oracle / test infrastructure only).

bf16 values are carried as float32 arrays whose low 16 mantissa bits are zero;
``round_bf16`` is IEEE round-to-nearest-even, the rounding torch applies when a
bf16 op stores its fp32 intermediate.
"""
from __future__ import annotations

import numpy as np


def round_bf16(x) -> np.ndarray:
    """Round to the nearest bfloat16 (ties to even); NaN stays NaN."""
    shape = np.shape(x)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(shape)
    u = np.ascontiguousarray(x).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).reshape(shape)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, x, out)
    return out


def to_bits(x) -> np.ndarray:
    """bf16-valued float32 array -> uint16 bit patterns."""
    x = round_bf16(x)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def from_bits(b) -> np.ndarray:
    """uint16 bit patterns -> float32 array of the bf16 values."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def rel_fro(a, b, eps: float = 1e-12) -> float:
    """‖a − b‖_F / max(‖b‖_F, eps) in float64 (the reference's rel_l2, hft.py:56-58)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), eps))
