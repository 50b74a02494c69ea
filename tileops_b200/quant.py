"""Symmetric INT8 quantize / dequantize, per tensor and per channel, on sm_100a.

Drop-in for tileops/quant.py::

    q = clamp(round(x / scale), -128, 127)      # int8, round half to even (torch.round)
    x_hat = float(q) * scale

The division runs in fp32 on the upcast input, as the reference's kernels do
(backend/cuda/quant.py:32-105 read x and the fp32 scale into one fp32 expression). The
per-channel forms index the channel in place (``[outer, C, inner]`` view) instead of the
reference's permute-to-last copy (tileops/_shape.py:24-49); results are identical.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _validate_scale_tensor(scale: torch.Tensor, *, op: str, numel: int = 1) -> torch.Tensor:
    """quant.py:36-50 (same checks, messages and exception types)."""
    if scale.dtype != torch.float32:
        raise TypeError(f"{op}: scale must be float32 (got {scale.dtype})")
    if scale.numel() != numel:
        raise ValueError(f"{op}: scale must have {numel} element(s), got {scale.numel()}")
    # The value check reads the device tensor back (a host sync), as the reference does; inside
    # a CUDA graph capture, where a sync is not allowed, the values are the caller's contract.
    if not (scale.is_cuda and torch.cuda.is_current_stream_capturing()) and torch.any(scale <= 0):
        raise ValueError(f"{op}: scale values must be positive")
    return scale.contiguous().reshape(numel)


def _channel_view(shape: torch.Size, dim: int, op: str) -> tuple[int, int, int]:
    nd = len(shape)
    if not 0 <= dim < nd:
        raise ValueError(f"{op}: invalid dim {dim} for ndim={nd}")
    c = shape[dim]
    if c <= 0:
        raise ValueError(f"{op}: reduced axis must have positive extent")
    outer = 1
    for s in shape[:dim]:
        outer *= s
    inner = 1
    for s in shape[dim + 1:]:
        inner *= s
    return outer, c, inner


def quantize_per_tensor(
    x: torch.Tensor,
    scale: torch.Tensor,
    *,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Quantize *x* with one scalar fp32 *scale* -> int8 (quant.py:53-93)."""
    op = "quantize_per_tensor"
    if not x.dtype.is_floating_point:
        raise TypeError(f"{op}: input must be floating-point (got {x.dtype})")
    sf = _validate_scale_tensor(scale, op=op, numel=1)
    if sf.device != x.device:
        raise TypeError(f"{op}: scale device must match input")
    _lib.ensure_device(x, op)
    xd = _lib.dtype_code(x.dtype, op)
    if out is not None:
        if out.shape != x.shape or out.dtype != torch.int8:
            raise ValueError(f"{op}: out must be int8 with shape {tuple(x.shape)}")
        if out.device != x.device:
            raise TypeError(f"{op}: out device must match input")
    xc = x.contiguous()
    dst = out if (out is not None and out.is_contiguous()) else torch.empty(
        x.shape, dtype=torch.int8, device=x.device)
    _lib.call("to_quant_per_tensor_i8", xc.data_ptr(), xd, sf.data_ptr(), dst.data_ptr(),
              xc.numel(), _lib.stream_ptr())
    if out is not None:
        if dst is not out:
            out.copy_(dst)
        return out
    return dst


def dequantize_per_tensor(
    x_q: torch.Tensor,
    scale: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.float32,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Dequantize int8 *x_q* with a scalar *scale* (quant.py:96-141)."""
    op = "dequantize_per_tensor"
    if x_q.dtype != torch.int8:
        raise TypeError(f"{op}: input must be torch.int8 (got {x_q.dtype})")
    if out_dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise TypeError(f"{op}: out_dtype must be float32, float16, or bfloat16")
    sf = _validate_scale_tensor(scale, op=op, numel=1)
    if sf.device != x_q.device:
        raise TypeError(f"{op}: scale device must match input")
    _lib.ensure_device(x_q, op)
    if out is None:
        dst = torch.empty(x_q.shape, dtype=out_dtype, device=x_q.device)
    else:
        if out.shape != x_q.shape or out.dtype != out_dtype:
            raise ValueError(f"{op}: out must be {out_dtype} with shape {tuple(x_q.shape)}")
        if out.device != x_q.device:
            raise TypeError(f"{op}: out device must match input")
        dst = out if out.is_contiguous() else torch.empty_like(out, memory_format=torch.contiguous_format)
    qc = x_q.contiguous()
    _lib.call("to_dequant_per_tensor_i8", qc.data_ptr(), sf.data_ptr(), dst.data_ptr(),
              _lib.DTYPE_CODES[out_dtype], qc.numel(), _lib.stream_ptr())
    if out is not None and dst is not out:
        out.copy_(dst)
        return out
    return dst


def quantize_per_channel(
    x: torch.Tensor,
    scale: torch.Tensor,
    dim: int,
    *,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Quantize *x* with one fp32 scale per index along *dim* (quant.py:144-190)."""
    op = "quantize_per_channel"
    if not x.dtype.is_floating_point:
        raise TypeError(f"{op}: input must be floating-point (got {x.dtype})")
    dim = dim if dim >= 0 else dim + x.ndim
    n = x.shape[dim]
    sf = _validate_scale_tensor(scale, op=op, numel=n)
    if sf.device != x.device:
        raise TypeError(f"{op}: scale device must match input")
    outer, c, inner = _channel_view(x.shape, dim, op)
    _lib.ensure_device(x, op)
    xd = _lib.dtype_code(x.dtype, op)
    if out is not None:
        if out.shape != x.shape or out.dtype != torch.int8:
            raise ValueError(f"{op}: out must be int8 with shape {tuple(x.shape)}")
        if out.device != x.device:
            raise TypeError(f"{op}: out device must match input")
    xc = x.contiguous()
    dst = out if (out is not None and out.is_contiguous()) else torch.empty(
        x.shape, dtype=torch.int8, device=x.device)
    _lib.call("to_quant_per_channel_i8", xc.data_ptr(), xd, sf.data_ptr(), dst.data_ptr(),
              outer, c, inner, _lib.stream_ptr())
    if out is not None:
        if dst is not out:
            out.copy_(dst)
        return out
    return dst


def dequantize_per_channel(
    x_q: torch.Tensor,
    scale: torch.Tensor,
    dim: int,
    *,
    out_dtype: torch.dtype = torch.float32,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Dequantize int8 *x_q* with per-channel *scale* along *dim* (quant.py:193-248)."""
    op = "dequantize_per_channel"
    if x_q.dtype != torch.int8:
        raise TypeError(f"{op}: input must be torch.int8 (got {x_q.dtype})")
    if out_dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise TypeError(f"{op}: out_dtype must be float32, float16, or bfloat16")
    dim = dim if dim >= 0 else dim + x_q.ndim
    n = x_q.shape[dim]
    sf = _validate_scale_tensor(scale, op=op, numel=n)
    if sf.device != x_q.device:
        raise TypeError(f"{op}: scale device must match input")
    outer, c, inner = _channel_view(x_q.shape, dim, op)
    _lib.ensure_device(x_q, op)
    if out is None:
        dst = torch.empty(x_q.shape, dtype=out_dtype, device=x_q.device)
    else:
        if out.shape != x_q.shape or out.dtype != out_dtype:
            raise ValueError(f"{op}: out must be {out_dtype} with shape {tuple(x_q.shape)}")
        if out.device != x_q.device:
            raise TypeError(f"{op}: out device must match input")
        dst = out if out.is_contiguous() else torch.empty_like(out, memory_format=torch.contiguous_format)
    qc = x_q.contiguous()
    _lib.call("to_dequant_per_channel_i8", qc.data_ptr(), sf.data_ptr(), dst.data_ptr(),
              _lib.DTYPE_CODES[out_dtype], outer, c, inner, _lib.stream_ptr())
    if out is not None:
        if dst is not out:
            out.copy_(dst)
        return out
    return dst


__all__ = [
    "dequantize_per_channel",
    "dequantize_per_tensor",
    "quantize_per_channel",
    "quantize_per_tensor",
]
