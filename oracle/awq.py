"""AWQ W4A16 oracle (test infrastructure only) -- restates tileops/quant_awq.py."""

from __future__ import annotations

import numpy as np

from .numerics import rounder

# quant_awq.py:22 -- logical column i of a word sits in nibble ORDER[i].
REVERSE_AWQ_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)


def pack(unpacked: np.ndarray) -> np.ndarray:
    """quant_awq.py:55-65: [..., 8C] ints -> [..., C] int32 (low nibble of each value,
    built in 64-bit then wrapped to int32)."""
    u = np.asarray(unpacked).astype(np.int64)
    if u.shape[-1] % 8:
        raise ValueError("pack_awq_int4: last dimension must be divisible by 8")
    t = u.reshape(*u.shape[:-1], u.shape[-1] // 8, 8)
    w = np.zeros(t.shape[:-1], dtype=np.int64)
    for i, sh in enumerate(REVERSE_AWQ_ORDER):
        w |= (t[..., i] & 0xF) << (4 * sh)
    return w.astype(np.uint32).view(np.int32) if w.size else w.astype(np.int32)


def unpack(packed: np.ndarray) -> np.ndarray:
    """quant_awq.py:41-52: [..., C] int32/int64 words -> [..., 8C] int64 nibbles."""
    w = np.asarray(packed).astype(np.int64)
    pieces = [(w >> (4 * sh)) & 0xF for sh in REVERSE_AWQ_ORDER]
    st = np.stack(pieces, axis=-1)
    return st.reshape(*w.shape[:-1], w.shape[-1] * 8)


def dequant(qweight: np.ndarray, scales_f32: np.ndarray, qzeros: np.ndarray, dtype: str) -> np.ndarray:
    """quant_awq.py:68-109: W[k, n] = dtype((w - z) * s), s and the result in ``dtype``
    ('f16', 'bf16' or 'f32'); ``scales_f32`` holds the scale values (exact in dtype)."""
    rnd = rounder(dtype)
    k = qweight.shape[0]
    g = scales_f32.shape[0]
    gs = k // g
    w = unpack(qweight).astype(np.float32)
    z = unpack(qzeros).astype(np.float32)
    gidx = np.arange(k) // gs
    return rnd((w - z[gidx]) * np.asarray(scales_f32, dtype=np.float32)[gidx])


def gemm(x_f32: np.ndarray, qweight, scales_f32, qzeros, dtype: str) -> np.ndarray:
    """quant_awq.py:112-155: y = dtype(x @ dequant(W)) with the sum carried in float64
    (the fp32-accumulated reference the parity tolerance is stated against)."""
    rnd = rounder(dtype)
    w = dequant(qweight, scales_f32, qzeros, dtype).astype(np.float64)
    x = rnd(np.asarray(x_f32, dtype=np.float32)).astype(np.float64)
    return rnd((x @ w).astype(np.float32))


def gemm_reference_cpu(x_f32, qweight, scales_f32, qzeros, dtype: str) -> np.ndarray:
    """The reference's CPU algorithm as it runs (dequantise the whole weight, then a dense
    fp32 matmul); timed as the CPU baseline."""
    rnd = rounder(dtype)
    w = dequant(qweight, scales_f32, qzeros, dtype)
    return rnd(rnd(np.asarray(x_f32, dtype=np.float32)) @ w)


def gemm_reference_cpu_torch(x, qweight, scales, qzeros, group_size):
    """The reference algorithm (quant_awq.py:41-52, 104-109, 153-155: int64 unpack of both
    packed tensors, per-row gathers of zeros and scales, (w - z) * s in scales.dtype, then a
    matmul in scales.dtype) restated on torch CPU tensors; timed as the CPU baseline."""
    import torch

    def unpack(p):
        w = p.to(torch.int64)
        pieces = [(w >> (4 * sh)) & 0xF for sh in REVERSE_AWQ_ORDER]
        return torch.stack(pieces, dim=-1).reshape(*p.shape[:-1], p.shape[-1] * 8)

    sd = scales.dtype
    k = qweight.shape[0]
    w = unpack(qweight).to(sd)
    z = unpack(qzeros).to(sd)
    gidx = torch.arange(k) // group_size
    weight = (w - z[gidx]) * scales[gidx]
    return x.to(sd) @ weight
