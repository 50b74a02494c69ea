"""Gated-activation oracle (test infrastructure only) -- restates the kernels of
tileops/fused.py:97-114 (tileops/backend/cuda/fused.py:17-29 silu, :32-46 gelu_tanh):
``C = act(A) * B`` element-wise, act evaluated in fp32, rounded to the tensor dtype, then the
product rounded again (the two roundings of ``F.silu(a) * b`` in the tensor dtype, which is
what the reference's tests/fused.py compares against).

Pinned by tests/golden/fused.npz (torch CPU ``F.silu(a) * b`` and
``F.gelu(a, approximate="tanh") * b``, the comparators of the reference's tests)."""

from __future__ import annotations

import numpy as np

from .numerics import rounder


def _silu(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def _gelu_tanh(x: np.ndarray) -> np.ndarray:
    inner = np.float32(0.7978845608028654) * (x + np.float32(0.044715) * x * x * x)
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(inner))).astype(np.float32)


def act_and_mul(a: np.ndarray, b: np.ndarray, act: str, dtype: str) -> np.ndarray:
    """fp32 values of ``act(a) * b`` for inputs holding ``dtype`` values ('f32', 'f16', 'bf16')."""
    rnd = rounder(dtype)
    a32 = np.asarray(a, np.float32)
    g = rnd(_silu(a32) if act == "silu" else _gelu_tanh(a32))
    return rnd(g.astype(np.float32) * np.asarray(b, np.float32))


def silu_and_mul(a, b, dtype: str) -> np.ndarray:
    return act_and_mul(a, b, "silu", dtype)


def gelu_and_mul(a, b, dtype: str) -> np.ndarray:
    return act_and_mul(a, b, "gelu", dtype)
