"""Gated activations of an MLP block, as in the reference's ``tileops.fused``
(tileops/fused.py:97-114): ``silu_and_mul(a, b)`` = ``silu(a) * b`` and ``gelu_and_mul(a, b)`` =
``gelu(a, tanh approximation) * b``, element-wise over same-shaped tensors, with the
reference's argument names, ``out=`` keyword and validation (ValueError for shapes and devices,
TypeError for dtypes).

Inputs may be strided views whose last dimension is contiguous (for example the gate and up
halves ``u[:, :F]`` and ``u[:, F:]`` of a fused gate_up output): the kernel reads them in place.
Other layouts are made contiguous first. An ``out`` that the kernel cannot write in place (a
transposed view, say) receives a copy of the result and is returned, as in the reference.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _validate_fused(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor],
                    op: str) -> None:
    # Same checks, order and messages as tileops/fused.py:34-64.
    if a.shape != b.shape:
        raise ValueError(f"{op}: shape mismatch — a.shape={a.shape}, b.shape={b.shape}")
    if a.dtype != b.dtype:
        raise TypeError(f"{op}: dtype mismatch — a.dtype={a.dtype}, b.dtype={b.dtype}")
    if a.device != b.device:
        raise ValueError(f"{op}: device mismatch — a.device={a.device}, b.device={b.device}")
    if out is not None:
        if out.shape != a.shape:
            raise ValueError(f"{op}: out.shape={out.shape} != input shape {a.shape}")
        if out.dtype != a.dtype:
            raise TypeError(f"{op}: out.dtype={out.dtype} != input dtype {a.dtype}")
        if out.device != a.device:
            raise ValueError(f"{op}: out.device={out.device} != input device {a.device}")


def _row_stride(t: torch.Tensor) -> Optional[int]:
    """Row stride of ``t`` seen as [numel / last, last] with a contiguous last dimension, or
    None when it cannot be seen that way without a copy."""
    if t.dim() == 0:
        return 1
    cols = t.shape[-1]
    if cols > 1 and t.stride(-1) != 1:
        return None
    if t.dim() == 1:
        return cols
    # the leading dimensions must collapse into one row index
    for i in range(t.dim() - 2):
        if t.shape[i] > 1 and t.stride(i) != t.stride(i + 1) * t.shape[i + 1]:
            return None
    if t.shape[-2] <= 1:
        return cols
    ld = t.stride(-2)
    return ld if ld >= cols else None


def _act_mul(op: str, entry: str, a: torch.Tensor, b: torch.Tensor,
             out: Optional[torch.Tensor]) -> torch.Tensor:
    _validate_fused(a, b, out, op)
    _lib.ensure_device(a, op)
    if a.dtype not in _DTYPES:
        raise TypeError(f"{op}: unsupported dtype {a.dtype} (float32, float16 and bfloat16 are "
                        "supported)")
    cols = a.shape[-1] if a.dim() > 0 else 1
    rows = a.numel() // cols if cols else 0
    lda = _row_stride(a)
    if lda is None:
        a = a.contiguous()
        lda = cols
    ldb = _row_stride(b)
    if ldb is None:
        b = b.contiguous()
        ldb = cols
    dst = out
    ldc = _row_stride(out) if out is not None else None
    if ldc is None:
        dst = torch.empty(a.shape, dtype=a.dtype, device=a.device)
        ldc = cols
    if a.numel():
        _lib.call(entry, a.data_ptr(), b.data_ptr(), dst.data_ptr(), _lib.DTYPE_CODES[a.dtype],
                  rows, cols, lda, ldb, ldc, _lib.stream_ptr())
    if out is not None and dst is not out:
        out.copy_(dst)
        return out
    return dst


def silu_and_mul(a: torch.Tensor, b: torch.Tensor, *,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(a) * b`` element-wise (same shapes) -- tileops/fused.py:97."""
    return _act_mul("silu_and_mul", "to_silu_and_mul", a, b, out)


def gelu_and_mul(a: torch.Tensor, b: torch.Tensor, *,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``gelu(a) * b`` with the tanh GELU approximation -- tileops/fused.py:107."""
    return _act_mul("gelu_and_mul", "to_gelu_and_mul", a, b, out)


def act_and_mul_group_quant(a: torch.Tensor, b: torch.Tensor, group_size: int, *,
                            act: str = "silu", dtype: Optional[torch.dtype] = None,
                            eps: float = 1e-10, column_major_scales: bool = False,
                            use_ue8m0: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Library extension (no reference counterpart): ``silu_and_mul(a, b)`` (or gelu with
    ``act="gelu"``) quantised per token group -- ``per_token_group_quant_fp8`` of it
    (tileops/quant_fp8.py:83; dtype ``torch.float8_e4m3fn``, the default) or
    ``per_token_group_quant_int8`` (tileops/quant_int8.py:109; dtype ``torch.int8``) -- in one
    kernel that never writes the activation. Returns the same ``(q, scales)`` as the two ops
    run one after the other, bit for bit: the input of a W8A8 down projection straight from
    the gate and up halves of the gate_up output."""
    op = "act_and_mul_group_quant"
    _validate_fused(a, b, None, op)
    if act not in ("silu", "gelu"):
        raise ValueError(f"{op}: act must be 'silu' or 'gelu' (got {act!r})")
    dtype = torch.float8_e4m3fn if dtype is None else dtype
    if dtype not in (torch.float8_e4m3fn, torch.int8):
        raise TypeError(f"{op}: codes must be torch.float8_e4m3fn or torch.int8 (got {dtype})")
    if dtype == torch.int8 and (use_ue8m0 or column_major_scales):
        raise ValueError(f"{op}: use_ue8m0 and column_major_scales are FP8 options")
    _lib.ensure_device(a, op)
    if a.dtype not in _DTYPES:
        raise TypeError(f"{op}: unsupported dtype {a.dtype} (float32, float16 and bfloat16 are "
                        "supported)")
    if a.dim() == 0 or a.shape[-1] % group_size != 0:
        raise ValueError(f"the last dimension of `a` must be divisible by `group_size` "
                         f"{group_size}")
    if column_major_scales and a.dim() != 2:
        raise ValueError(f"{op}: column_major_scales needs 2-D inputs")
    cols = a.shape[-1]
    rows = a.numel() // cols if cols else 0
    lda, ldb = _row_stride(a), _row_stride(b)
    if lda is None:
        a, lda = a.contiguous(), cols
    if ldb is None:
        b, ldb = b.contiguous(), cols
    q = torch.empty(a.shape, dtype=dtype, device=a.device)
    groups = cols // group_size
    s = torch.empty(*a.shape[:-1], groups, dtype=torch.float32, device=a.device)
    if a.numel():
        _lib.call("to_act_and_mul_group_quant", a.data_ptr(), b.data_ptr(),
                  _lib.DTYPE_CODES[a.dtype], rows, cols, lda, ldb, 0 if act == "silu" else 1,
                  group_size, eps, 1 if use_ue8m0 else 0, 1 if column_major_scales else 0,
                  _lib.DTYPE_CODES[dtype], q.data_ptr(), s.data_ptr(), _lib.stream_ptr())
    return q, s


__all__ = ["act_and_mul_group_quant", "gelu_and_mul", "silu_and_mul"]
