"""Dense GEMM and GEMV, as in the reference's ``tileops.gemm`` / ``tileops.mm``
(tileops/blas/gemm.py:31-78, out handling tileops/runtime/__init__.py:579-595) and
``tileops.gemv`` / ``tileops.mv`` (tileops/blas/gemv.py:22-67): ``C = A @ B`` with A (M, K) and
B (K, N) row-major, and ``y = A @ x``; fp32 accumulation, results in the inputs' dtype.

This is the dense comparator of the quantized layers: the same tcgen05 tiles as the W8A8 GEMMs
(kind::f16, A K-major, B read MN-major as 64-column strips, no scales). float16 and bfloat16
run on those tiles when K % 8 == 0 and N % 64 == 0 with 16-byte aligned operands; other
shapes, and float32, run on the library's SIMT tiles (fp32 FMA).
GEMV runs on its own streaming kernel for float32, float16 and bfloat16 at every shape.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def gemm(a: torch.Tensor, b: torch.Tensor, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Matrix multiply ``C = A @ B`` (2-D tensors, row-major) -- tileops/blas/gemm.py:31."""
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("gemm expects 2-D A and B")
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError(f"gemm: incompatible shapes {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.dtype != b.dtype:
        raise TypeError("gemm: A and B dtypes must match")
    if a.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        # ValueError, as tileops/runtime/__init__.py:130 raises for a dtype outside these three
        raise ValueError(f"Unsupported dtype {a.dtype}; expected one of torch.float32, "
                         "torch.float16, torch.bfloat16")
    _lib.ensure_device(a, "gemm")
    _lib.same_device("gemm", a, b)
    aa = a.contiguous()
    bb = b.contiguous()
    if out is None:
        out = torch.empty(m, n, dtype=a.dtype, device=a.device)
    else:
        if out.shape != (m, n):
            raise ValueError(f"gemm: out.shape={tuple(out.shape)} != ({m}, {n})")
        if out.dtype != a.dtype or out.device != a.device:
            raise TypeError("gemm: out dtype/device must match A")
    cc = out.contiguous()
    _lib.call("to_gemm", aa.data_ptr(), bb.data_ptr(), cc.data_ptr(), _lib.DTYPE_CODES[a.dtype],
              m, n, k, _lib.stream_ptr())
    if cc.data_ptr() != out.data_ptr():
        out.copy_(cc)
    return out


def mm(input: torch.Tensor, mat2: torch.Tensor, *,
       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``torch.mm`` -- 2-D matrix multiply ``input @ mat2`` (tileops/blas/gemm.py:71)."""
    return gemm(input, mat2, out=out)


def gemv(a: torch.Tensor, x: torch.Tensor, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Matrix-vector multiply ``y = A @ x`` with A (M, K) and x (K,) -- tileops/blas/gemv.py:22.

    fp32 accumulation on the streaming kernel for float32, float16 and bfloat16; y in the
    inputs' dtype. Argument checks and ``out`` handling follow tileops/blas/gemv.py:32-41 and
    tileops/runtime/__init__.py:627-641.
    """
    if a.ndim != 2 or x.ndim != 1:
        raise ValueError("gemv expects A 2-D and x 1-D")
    m, k = a.shape
    if x.shape[0] != k:
        raise ValueError(f"gemv: A.shape[1]={k} != len(x)={x.shape[0]}")
    if a.dtype != x.dtype:
        raise TypeError("gemv: A and x dtypes must match")
    if a.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        # ValueError, as tileops/runtime/__init__.py:130 raises for a dtype outside these three
        raise ValueError(f"Unsupported dtype {a.dtype}; expected one of torch.float32, "
                         "torch.float16, torch.bfloat16")
    _lib.ensure_device(a, "gemv")
    _lib.same_device("gemv", a, x)
    aa = a.contiguous()
    xx = x.contiguous()
    if out is None:
        out = torch.empty(m, dtype=a.dtype, device=a.device)
    else:
        if out.shape != (m,):
            raise ValueError(f"gemv: out.shape={tuple(out.shape)} != ({m},)")
        if out.dtype != a.dtype or out.device != a.device:
            raise TypeError("gemv: out dtype/device must match A")
    yy = out.contiguous()
    _lib.call("to_gemv", aa.data_ptr(), xx.data_ptr(), yy.data_ptr(), _lib.DTYPE_CODES[a.dtype],
              m, k, _lib.stream_ptr())
    if yy.data_ptr() != out.data_ptr():
        out.copy_(yy)
    return out


def mv(input: torch.Tensor, vec: torch.Tensor, *,
       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``torch.mv`` -- matrix-vector ``input @ vec`` (tileops/blas/gemv.py:60)."""
    return gemv(input, vec, out=out)


__all__ = ["gemm", "gemv", "mm", "mv"]
