"""INT8 W8A8 oracle (test infrastructure only) -- restates tileops/quant_int8.py."""

from __future__ import annotations

import numpy as np

from .numerics import rounder


def input_to_int8(x_f32: np.ndarray, dtype: str):
    """quant_int8.py:29-40, evaluated in ``dtype`` as torch does for a tensor of that dtype:
    amax = T(max(amax, 1e-12)); s = T(T(1 / amax) * 127)  (``127 / amax`` is
    ``amax.reciprocal() * 127`` in torch); q = int8(trunc(clamp(T(x * s), -128, 127)));
    returns (q, float32(1 / s))."""
    rnd = rounder(dtype)
    x = rnd(np.asarray(x_f32, dtype=np.float32))
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0)
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        # In float16, 1e-12 rounds to 0: an all-zero tensor divides by zero (s = inf) and
        # 0 * inf is NaN, which torch's clamp keeps and its int8 cast turns into 0.
        amax = rnd(np.maximum(amax, np.float32(1e-12)))
        r = rnd(np.float32(1.0) / amax)
        s = rnd(np.float32(r) * np.float32(127.0))
        y = rnd(x * np.float32(s))
        nan = np.isnan(y)
        y = np.clip(np.where(nan, np.float32(0), y), -128.0, 127.0)
        q = np.trunc(y).astype(np.int8)
        return q, np.float32(np.float32(1.0) / np.float32(s))


def group_quant(x_f32: np.ndarray, group_size: int, eps: float = 1e-10):
    """quant_int8.py:43-51 applied per group (quant_int8.py:109-133, per-token = group K):
    scale = max(absmax, eps) / 127 (fp32), q = clamp(round_half_even(x / scale), -128, 127).
    Returns q with x's shape and scales [..., K / G]."""
    x = np.asarray(x_f32, dtype=np.float32)
    lead, k = x.shape[:-1], x.shape[-1]
    flat = x.reshape(-1, group_size)
    absmax = np.maximum(np.max(np.abs(flat), axis=-1), np.float32(eps)) if flat.size else \
        np.zeros(flat.shape[0], np.float32)
    scale = (absmax / np.float32(127.0)).astype(np.float32)
    with np.errstate(invalid="ignore"):
        y = np.rint(flat / scale[:, None])
    q = np.clip(np.where(np.isnan(y), np.float32(0), y), -128, 127).astype(np.int8)  # NaN in: 0
    return q.reshape(*lead, k), scale.reshape(*lead, k // group_size)


def block_dequant(q: np.ndarray, s: np.ndarray, block_size) -> np.ndarray:
    """quant_int8.py:136-159: y[n, k] = float32(q[n, k]) * s[n // bn, k // bk]."""
    bn, bk = block_size
    n, k = q.shape
    rows = np.arange(n) // bn
    cols = np.arange(k) // bk
    return (q.astype(np.float32) * np.asarray(s, np.float32)[rows][:, cols]).astype(np.float32)


def accumulators(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact integer sum_k A[m,k] * B[n,k]. Evaluated as a float64 GEMM, exact while
    |sum| < 2^53 (K * 127^2 for these shapes)."""
    assert a.shape[-1] * 128 * 128 < 2 ** 53
    return (a.astype(np.float64) @ b.astype(np.float64).T).astype(np.int64)


def block_matmul(a: np.ndarray, b: np.ndarray, a_s: np.ndarray, b_s: np.ndarray, block_size,
                 out_dtype: str) -> np.ndarray:
    """quant_int8.py:180-228, C = dequant(A) @ dequant(B).T -> out_dtype, with exact integer
    block sums scaled in float64 (the fp32-accumulated reference of the tolerance)."""
    bn, bk = block_size
    m, k = a.shape
    n = b.shape[0]
    kt = -(-k // bk)
    acc = np.zeros((m, n), dtype=np.float64)
    rows_b = np.arange(n) // bn
    for kb in range(kt):
        sl = slice(kb * bk, min(k, (kb + 1) * bk))
        part = a[:, sl].astype(np.float64) @ b[:, sl].astype(np.float64).T
        acc += part * a_s[:, kb].astype(np.float64)[:, None] * b_s[rows_b, kb].astype(np.float64)[None, :]
    return rounder(out_dtype)(acc.astype(np.float32))


def block_matmul_reference_cpu(a, b, a_s, b_s, block_size, out_dtype: str) -> np.ndarray:
    """The reference's CPU algorithm as it runs (fp32 dequant of both operands, then an fp32
    GEMM); timed as the CPU baseline."""
    bn, bk = block_size
    m, k = a.shape
    cols = np.arange(k) // bk
    a_f = a.astype(np.float32) * a_s.astype(np.float32)[:, cols]
    b_f = block_dequant(b, b_s, block_size)
    return rounder(out_dtype)(a_f @ b_f.T)


def block_matmul_reference_cpu_torch(a, b, a_s, b_s, block_size, out_dtype):
    """The reference algorithm (quant_int8.py:223-228: fp32 dequant of both operands, fp32
    GEMM, cast) on torch CPU tensors, the library the reference itself runs on; used as the
    timed CPU baseline because it is the fastest faithful CPU restatement available."""
    import torch

    bn, bk = block_size
    k = a.shape[1]
    cols = torch.arange(k) // bk
    rows = torch.arange(b.shape[0]) // bn
    a_f = a.to(torch.float32) * a_s.to(torch.float32)[:, cols]
    b_f = b.to(torch.float32) * b_s.to(torch.float32)[rows][:, cols]
    return (a_f @ b_f.T).to(out_dtype)
