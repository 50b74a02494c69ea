"""FP8 e4m3 facade: dynamic quantisation and block-scaled W8A8 FP8 matmul on sm_100a.

Drop-in for tileops/quant_fp8.py (names, arguments, dequant-scale convention, UE8M0 option,
column-major scale layout and error types). The quantisers and block_dequant take both
``torch.float8_e4m3fn`` and ``torch.float8_e4m3fnuz`` (the reference's ``dtype`` argument);
the W8A8 GEMMs take e4m3fn only -- sm_100's tensor cores have no e4m3fnuz operand -- and raise
NotImplementedError for e4m3fnuz.
"""

from __future__ import annotations

import math
from typing import Optional, Union

import torch

from . import _lib
from .quant_int8 import _FLOATS, _run_w8a8, _validate_w8a8, _validate_w8a8_rest

_FP8_DTYPES = tuple(
    d for d in (getattr(torch, "float8_e4m3fn", None), getattr(torch, "float8_e4m3fnuz", None))
    if d is not None
)


def is_fp8(x: Union[torch.dtype, torch.Tensor]) -> bool:
    """Whether *x* is an FP8 dtype or a tensor stored in FP8 (quant_fp8.py:25-29)."""
    if isinstance(x, torch.Tensor):
        x = x.dtype
    return x in _FP8_DTYPES


def default_fp8_dtype() -> torch.dtype:
    """``float8_e4m3fn`` (quant_fp8.py:32-36)."""
    if not _FP8_DTYPES:
        raise RuntimeError("PyTorch build has no float8_e4m3fn support")
    return _FP8_DTYPES[0]


def get_fp8_min_max(dtype: Optional[torch.dtype] = None) -> tuple[float, float]:
    """FP8 clamp bounds, with the FNUZ override to +-224 (quant_fp8.py:39-45)."""
    dtype = dtype if dtype is not None else default_fp8_dtype()
    if dtype == getattr(torch, "float8_e4m3fnuz", None):
        return -224.0, 224.0
    finfo = torch.finfo(dtype)
    return finfo.min, finfo.max


def _require_e4m3fn(dtype: torch.dtype, op: str) -> None:
    if dtype != torch.float8_e4m3fn:
        raise NotImplementedError(f"{op}: only torch.float8_e4m3fn is supported on sm_100 "
                                  f"(got {dtype})")


_FNUZ = getattr(torch, "float8_e4m3fnuz", None)


def _entry(dtype: torch.dtype, op: str, base: str) -> str:
    """The C entry of `base` for an FP8 code dtype: e4m3fn, or its _fnuz form."""
    if dtype == torch.float8_e4m3fn:
        return base
    if _FNUZ is not None and dtype == _FNUZ:
        return base + "_fnuz"
    raise NotImplementedError(f"{op}: unsupported FP8 dtype {dtype}")


def input_to_float8(
    x: torch.Tensor,
    dtype: Optional[torch.dtype] = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Tensor-wide dynamic quant -> ``(q, dequant_scale)`` (quant_fp8.py:52-63), arithmetic in
    ``x.dtype``: ``s = (1/amax) * fmax``, ``q = fp8(clamp(x * s, +-fmax))`` with fmax =
    finfo(dtype).max (448 for e4m3fn, 240 for e4m3fnuz)."""
    op = "input_to_float8"
    dtype = dtype if dtype is not None else default_fp8_dtype()
    entry = _entry(dtype, op, "to_input_to_fp8")
    _lib.ensure_device(x, op)
    if x.dtype not in _FLOATS:
        raise TypeError(f"{op}: unsupported input dtype {x.dtype}")
    if x.numel() == 0:
        raise RuntimeError(f"{op}: cannot compute amax of an empty tensor")
    xc = x.contiguous()
    q = torch.empty(x.shape, dtype=dtype, device=x.device)
    s = torch.empty((), dtype=torch.float32, device=x.device)
    ws_bytes = _lib.workspace_bytes("to_input_quant_workspace_size")
    ws = _lib.workspace(ws_bytes, x.get_device())
    _lib.call(entry, xc.data_ptr(), _lib.DTYPE_CODES[x.dtype], xc.numel(),
              q.data_ptr(), s.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_ptr())
    return q, s


def per_token_group_quant_fp8(
    x: torch.Tensor,
    group_size: int,
    eps: float = 1e-10,
    dtype: Optional[torch.dtype] = None,
    column_major_scales: bool = False,
    tma_aligned_scales: bool = False,
    out_q: Optional[torch.Tensor] = None,
    use_ue8m0: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token-group dynamic FP8 quant along the last dim (quant_fp8.py:83-140):
    ``scale = max(absmax, eps) / fmax`` (optionally rounded up to a power of two),
    ``q = fp8(clamp(x / scale, +-fmax))`` with get_fp8_min_max's fmax (448 for e4m3fn, 224
    for e4m3fnuz)."""
    if tma_aligned_scales:
        raise NotImplementedError(
            "per_token_group_quant_fp8: tma_aligned_scales is not implemented "
            "(use vLLM CUDA packed path for DeepGEMM TMA layouts)"
        )
    dtype = dtype if dtype is not None else default_fp8_dtype()
    if not is_fp8(dtype):
        raise TypeError(f"per_token_group_quant_fp8: unsupported dtype {dtype}")
    if x.shape[-1] % group_size != 0:
        raise ValueError(
            f"the last dimension of `x` {x.shape[-1]} must be divisible "
            f"by `group_size` {group_size}"
        )
    if x.stride(-1) != 1:
        raise ValueError("`x` groups must be contiguous along the last dimension")
    op = "per_token_group_quant_fp8"
    entry = _entry(dtype, op, "to_per_token_group_quant_fp8")
    _lib.ensure_device(x, op)
    if x.dtype not in _FLOATS:
        raise TypeError(f"{op}: unsupported input dtype {x.dtype}")
    if not x.is_contiguous():
        x = x.contiguous()
    if out_q is not None and (out_q.shape != x.shape or out_q.dtype != dtype):
        raise ValueError(
            f"per_token_group_quant_fp8: out_q must be {dtype} with shape {tuple(x.shape)}"
        )
    if column_major_scales and x.dim() < 2:
        raise ValueError("per_token_group_quant_fp8: column_major_scales requires ndim >= 2")
    _lib.same_device(op, x, out_q)
    lead = x.shape[:-1]
    k = x.shape[-1]
    num_groups = k // group_size
    n_groups = x.numel() // group_size if group_size else 0
    direct = out_q is not None and out_q.is_contiguous()
    q = out_q if direct else torch.empty(x.shape, dtype=dtype, device=x.device)
    if column_major_scales:
        # The reference returns s_flat.reshape(..., G_, M).transpose(-2, -1).contiguous()
        # (quant_fp8.py:134-136); the kernel writes that contiguous [..., M, G_] tensor.
        m = x.shape[-2]
        x_s = torch.empty(*x.shape[:-2], m, num_groups, dtype=torch.float32, device=x.device)
        cm_rows, cm_groups = m, num_groups
    else:
        x_s = torch.empty(*lead, num_groups, dtype=torch.float32, device=x.device)
        cm_rows, cm_groups = 0, 0
    _lib.call(entry, x.data_ptr(), _lib.DTYPE_CODES[x.dtype], n_groups,
              group_size, eps, 1 if use_ue8m0 else 0, cm_rows, cm_groups, q.data_ptr(),
              x_s.data_ptr(), _lib.stream_ptr())
    if out_q is not None and not direct:
        out_q.copy_(q)
        q = out_q
    return q, x_s


def per_token_group_quant_fp8_tma_aligned(
    x: torch.Tensor,
    group_size: int,
    eps: float = 1e-10,
    use_ue8m0: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Library extension: ``per_token_group_quant_fp8`` of a 2-D ``x`` [M, K] (e4m3fn codes)
    with the scales in the TMA-aligned column-major layout that the reference's
    ``tma_aligned_scales=True`` leaves unimplemented (quant_fp8.py:94-98): a [M, K/G] view with
    strides (1, ld), ld = M rounded up to 4, so every group's column of scales starts 16-byte
    aligned for a TMA load. Same codes and scale values as per_token_group_quant_fp8."""
    op = "per_token_group_quant_fp8"
    if x.dim() != 2:
        raise ValueError(f"{op}: TMA-aligned scales need a 2-D input")
    if x.shape[-1] % group_size != 0:
        raise ValueError(
            f"the last dimension of `x` {x.shape[-1]} must be divisible "
            f"by `group_size` {group_size}"
        )
    _lib.ensure_device(x, op)
    if x.dtype not in _FLOATS:
        raise TypeError(f"{op}: unsupported input dtype {x.dtype}")
    x = x.contiguous()
    m, k = x.shape
    groups = k // group_size
    ld = (m + 3) // 4 * 4
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    buf = torch.empty(groups, ld, dtype=torch.float32, device=x.device)
    _lib.call("to_per_token_group_quant_fp8_tma", x.data_ptr(), _lib.DTYPE_CODES[x.dtype], m, k,
              group_size, eps, 1 if use_ue8m0 else 0, q.data_ptr(), buf.data_ptr(), ld,
              _lib.stream_ptr())
    return q, buf.t()[:m]


def block_dequant(
    x_q_block: torch.Tensor,
    x_s: torch.Tensor,
    block_size: list[int],
) -> torch.Tensor:
    """Block-wise dequantisation of a 2-D FP8 weight -> fp32 (quant_fp8.py:143-168)."""
    if not is_fp8(x_q_block):
        raise TypeError(f"block_dequant: expected FP8 weights, got {x_q_block.dtype}")
    block_n, block_k = block_size[0], block_size[1]
    n, k = x_q_block.shape
    n_tiles = (n + block_n - 1) // block_n
    k_tiles = (k + block_k - 1) // block_k
    if n_tiles != x_s.shape[0] or k_tiles != x_s.shape[1]:
        raise ValueError(
            f"block_dequant: scale shape {tuple(x_s.shape)} does not match "
            f"block grid ({n_tiles}, {k_tiles}) for {tuple(x_q_block.shape)}"
        )
    op = "block_dequant"
    entry = _entry(x_q_block.dtype, op, "to_block_dequant_fp8")
    _lib.ensure_device(x_q_block, op)
    _lib.same_device(op, x_q_block, x_s)
    q = x_q_block.contiguous()
    s = x_s.to(torch.float32).contiguous()
    y = torch.empty(n, k, dtype=torch.float32, device=q.device)
    _lib.call(entry, q.data_ptr(), s.data_ptr(), y.data_ptr(), n, k, block_n,
              block_k, _lib.stream_ptr())
    return y


def _dequant_per_token_group_lastdim(
    a_q: torch.Tensor,
    a_s: torch.Tensor,
    group_k: int,
) -> torch.Tensor:
    """``A_f[..., k] = a_q[..., k] * a_s[..., k // group_k]`` in fp32 (quant_fp8.py:171-185)."""
    k = a_q.shape[-1]
    m = a_q.numel() // k if k else 0
    y = block_dequant(a_q.reshape(m, k), a_s.reshape(m, -1), [1, group_k])
    return y.view(*a_q.shape)


def w8a8_block_fp8_matmul(
    a: torch.Tensor,
    b: torch.Tensor,
    a_s: torch.Tensor,
    b_s: torch.Tensor,
    block_size: list[int],
    output_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """W8A8 FP8 block matmul ``C = dequant(A) @ dequant(B).T`` (quant_fp8.py:188-236) with
    e4m3 x e4m3 products accumulated in fp32 and the block scales applied per k-block."""
    op = "w8a8_block_fp8_matmul"
    block_n, block_k = _validate_w8a8(op, a, b, a_s, b_s, block_size)
    if not is_fp8(a) or not is_fp8(b):
        raise TypeError("w8a8_block_fp8_matmul: A and B must be FP8")
    m, n, k = _validate_w8a8_rest(op, a, b, a_s, b_s, block_n, block_k)
    _require_e4m3fn(a.dtype, op)
    _require_e4m3fn(b.dtype, op)
    return _run_w8a8("to_w8a8_fp8_gemm", op, a, b, a_s, b_s, block_n, block_k, m, n, k,
                     output_dtype)


def w8a8_triton_block_scaled_mm(
    a: torch.Tensor,
    b: torch.Tensor,
    a_s: torch.Tensor,
    b_s: torch.Tensor,
    block_size: list[int],
    output_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """vLLM name alias for :func:`w8a8_block_fp8_matmul` (quant_fp8.py:239-250)."""
    return w8a8_block_fp8_matmul(a, b, a_s, b_s, block_size, output_dtype=output_dtype)


def apply_w8a8_block_fp8_linear(
    input: torch.Tensor,
    weight: torch.Tensor,
    block_size: list[int],
    weight_scale: torch.Tensor,
    input_scale: Optional[torch.Tensor] = None,
    bias: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Group-quant the input, block FP8 matmul, add bias (quant_fp8.py:253-278)."""
    if input_scale is not None:
        raise ValueError("apply_w8a8_block_fp8_linear: input_scale must be None")
    input_2d = input.view(-1, input.shape[-1])
    output_shape = [*input.shape[:-1], weight.shape[0]]
    q_input, x_scale = per_token_group_quant_fp8(input_2d, block_size[1])
    op = "w8a8_block_fp8_matmul"
    block_n, block_k = _validate_w8a8(op, q_input, weight, x_scale, weight_scale, block_size)
    if not is_fp8(weight):
        raise TypeError("w8a8_block_fp8_matmul: A and B must be FP8")
    m, n, k = _validate_w8a8_rest(op, q_input, weight, x_scale, weight_scale, block_n, block_k)
    _require_e4m3fn(weight.dtype, op)
    fuse = bias is not None and bias.dtype == input.dtype and bias.numel() == n
    output = _run_w8a8("to_w8a8_fp8_gemm", op, q_input, weight, x_scale, weight_scale, block_n,
                       block_k, m, n, k, input.dtype, bias=bias.contiguous() if fuse else None)
    if bias is not None and not fuse:
        output = output + bias
    return output.to(dtype=input.dtype).view(*output_shape)


__all__ = [
    "apply_w8a8_block_fp8_linear",
    "block_dequant",
    "default_fp8_dtype",
    "get_fp8_min_max",
    "input_to_float8",
    "is_fp8",
    "per_token_group_quant_fp8",
    "per_token_group_quant_fp8_tma_aligned",
    "w8a8_block_fp8_matmul",
    "w8a8_triton_block_scaled_mm",
]
