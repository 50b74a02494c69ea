"""Symmetric INT8 oracle (test infrastructure only) -- restates tileops/quant.py and the
expressions of its kernels (tileops/backend/cuda/quant.py:32-105) with torch.round's
half-to-even rounding, as the reference's tests pin it (tests/quant.py:18-43)."""

from __future__ import annotations

import numpy as np

from .numerics import rounder


def _scale_view(scale, ndim: int, dim: int):
    s = np.asarray(scale, np.float32).reshape(-1)
    if dim is None:
        return np.float32(s[0])
    shape = [1] * ndim
    shape[dim] = -1
    return s.reshape(shape)


def quantize(x_f32: np.ndarray, scale, dim=None) -> np.ndarray:
    """q = clamp(round_half_even(float32(x) / scale), -128, 127) (quant.py:53, :144)."""
    x = np.asarray(x_f32, np.float32)
    d = None if dim is None else (dim if dim >= 0 else dim + x.ndim)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = np.rint((x / _scale_view(scale, x.ndim, d)).astype(np.float32))
    # a zero scale gives +-inf (clamped to 127 / -128) and, for x = 0, NaN: torch's clamp keeps
    # it and its int8 cast makes it 0
    return np.clip(np.where(np.isnan(y), np.float32(0), y), -128, 127).astype(np.int8)


def dequantize(q: np.ndarray, scale, out_dtype: str, dim=None) -> np.ndarray:
    """x_hat = out_dtype(float32(q) * scale) (quant.py:96, :193)."""
    q = np.asarray(q)
    d = None if dim is None else (dim if dim >= 0 else dim + q.ndim)
    return rounder(out_dtype)((q.astype(np.float32) * _scale_view(scale, q.ndim, d)).astype(np.float32))
