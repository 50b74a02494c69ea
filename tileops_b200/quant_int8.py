"""INT8 W8A8 facade: dynamic INT8 quantisation and block-scaled W8A8 matmul on sm_100a.

Drop-in for tileops/quant_int8.py (same names, arguments, shapes, dequant-scale
convention ``absmax / 127`` and error types). The per-token quantiser is one kernel pass
(the reference runs a one-thread-per-row TileLang kernel, backend/cuda/quant.py:113-137),
and the matmul keeps exact int32 accumulators on the tensor cores instead of dequantising
both operands to fp32.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib

_FLOATS = (torch.float32, torch.float16, torch.bfloat16)


def input_to_int8(
    x: torch.Tensor,
    dtype: torch.dtype = torch.int8,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Tensor-wide dynamic quant -> ``(q, dequant_scale)`` (quant_int8.py:29-40).

    Arithmetic in ``x.dtype`` as the reference evaluates it: ``s = (1/amax) * 127``,
    ``q = trunc(clamp(x * s, -128, 127))``; the returned scale is ``1/float(s)``."""
    op = "input_to_int8"
    if dtype != torch.int8:
        raise NotImplementedError(f"{op}: only torch.int8 output is supported (got {dtype})")
    _lib.ensure_device(x, op)
    if x.dtype not in _FLOATS:
        raise TypeError(f"{op}: unsupported input dtype {x.dtype}")
    if x.numel() == 0:
        raise RuntimeError(f"{op}: cannot compute amax of an empty tensor")
    xc = x.contiguous()
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty((), dtype=torch.float32, device=x.device)
    ws_bytes = _lib.workspace_bytes("to_input_quant_workspace_size")
    ws = _lib.workspace(ws_bytes, x.get_device())
    _lib.call("to_input_to_int8", xc.data_ptr(), _lib.DTYPE_CODES[x.dtype], xc.numel(),
              q.data_ptr(), s.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_ptr())
    return q, s


def _group_quant_int8(x2: torch.Tensor, group_size: int, eps: float):
    """Runs the group quantiser over a contiguous tensor whose numel is a multiple of G."""
    n_groups = x2.numel() // group_size
    q = torch.empty(x2.shape, dtype=torch.int8, device=x2.device)
    s = torch.empty(n_groups, dtype=torch.float32, device=x2.device)
    _lib.call("to_per_token_group_quant_i8", x2.data_ptr(), _lib.DTYPE_CODES[x2.dtype], n_groups,
              group_size, eps, q.data_ptr(), s.data_ptr(), _lib.stream_ptr())
    return q, s


def per_token_quant_int8(
    x: torch.Tensor,
    eps: float = 1e-10,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row dynamic quant on the last dim; scales have trailing size 1
    (quant_int8.py:54-106): ``scale = max(absmax, eps) / 127``, ``q = round(x / scale)``."""
    op = "per_token_quant_int8"
    _lib.ensure_device(x, op)
    if x.dtype not in _FLOATS:
        raise TypeError(f"{op}: unsupported input dtype {x.dtype}")
    original_shape = x.shape
    if x.dim() == 1:
        x2 = x.unsqueeze(0)
        squeezed = True
    elif x.dim() > 2:
        x2 = x.reshape(-1, original_shape[-1])
        squeezed = False
    else:
        x2 = x
        squeezed = False
    k = x2.shape[-1]
    m = x2.shape[0]
    x2 = x2.contiguous()
    if k == 0:
        raise ValueError(f"{op}: last dimension must be non-empty")
    q, s = _group_quant_int8(x2, k, eps)
    s = s.view(m, 1)
    if squeezed:
        return q.squeeze(0), s.squeeze(0)
    return q.view(*original_shape), s.view(*original_shape[:-1], 1)


def per_token_group_quant_int8(
    x: torch.Tensor,
    group_size: int,
    eps: float = 1e-10,
    dtype: torch.dtype = torch.int8,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token-group dynamic quant along the last dim (quant_int8.py:109-133)."""
    if dtype != torch.int8:
        raise TypeError("per_token_group_quant_int8: only torch.int8 output is supported")
    if x.shape[-1] % group_size != 0:
        raise ValueError("the last dimension of `x` cannot be divisible by `group_size`")
    op = "per_token_group_quant_int8"
    _lib.ensure_device(x, op)
    if x.dtype not in _FLOATS:
        raise TypeError(f"{op}: unsupported input dtype {x.dtype}")
    x = x.contiguous()
    lead = x.shape[:-1]
    k = x.shape[-1]
    q, s = _group_quant_int8(x, group_size, eps)
    return q.view(*lead, k), s.view(*lead, k // group_size)


def _check_block_grid(x_q: torch.Tensor, x_s: torch.Tensor, block_size) -> tuple[int, int]:
    block_n, block_k = block_size[0], block_size[1]
    n, k = x_q.shape
    n_tiles = (n + block_n - 1) // block_n
    k_tiles = (k + block_k - 1) // block_k
    if n_tiles != x_s.shape[0] or k_tiles != x_s.shape[1]:
        raise ValueError(
            f"block_dequant: scale shape {tuple(x_s.shape)} does not match "
            f"block grid ({n_tiles}, {k_tiles}) for {tuple(x_q.shape)}"
        )
    return block_n, block_k


def block_dequant(
    x_q_block: torch.Tensor,
    x_s: torch.Tensor,
    block_size: list[int],
) -> torch.Tensor:
    """Block-wise dequantisation of a 2-D int8 weight -> fp32 (quant_int8.py:136-159)."""
    op = "block_dequant"
    block_n, block_k = _check_block_grid(x_q_block, x_s, block_size)
    _lib.ensure_device(x_q_block, op)
    _lib.same_device(op, x_q_block, x_s)
    if x_q_block.dtype != torch.int8:
        raise TypeError(f"{op}: expected int8 weights, got {x_q_block.dtype}")
    n, k = x_q_block.shape
    q = x_q_block.contiguous()
    s = x_s.to(torch.float32).contiguous()
    y = torch.empty(n, k, dtype=torch.float32, device=q.device)
    _lib.call("to_block_dequant_i8", q.data_ptr(), s.data_ptr(), y.data_ptr(), n, k, block_n,
              block_k, _lib.stream_ptr())
    return y


def _dequant_per_token_group_lastdim(
    a_q: torch.Tensor,
    a_s: torch.Tensor,
    group_k: int,
) -> torch.Tensor:
    """``A_f[..., k] = a_q[..., k] * a_s[..., k // group_k]`` in fp32 (quant_int8.py:162-177),
    evaluated with the block-dequant kernel over the flattened rows."""
    k = a_q.shape[-1]
    m = a_q.numel() // k if k else 0
    a2 = a_q.reshape(m, k)
    s2 = a_s.reshape(m, -1)
    # One row per "block row": block_n = 1, the row's scales are its group scales.
    y = block_dequant(a2, s2, [1, group_k]) if a_q.dtype == torch.int8 else None
    if y is None:
        raise TypeError("_dequant_per_token_group_lastdim: expected int8 activations")
    return y.view(*a_q.shape)


def _validate_w8a8(op, a, b, a_s, b_s, block_size):
    """Checks of quant_int8.py:189-221 / quant_fp8.py:197-229, in the same order."""
    if len(block_size) != 2:
        raise ValueError("block_size must have length 2")
    block_n, block_k = block_size[0], block_size[1]
    if a.shape[-1] != b.shape[-1]:
        raise ValueError(f"{op}: K mismatch {a.shape[-1]} vs {b.shape[-1]}")
    return block_n, block_k


def _validate_w8a8_rest(op, a, b, a_s, b_s, block_n, block_k):
    if not a.is_contiguous() or not b.is_contiguous():
        raise ValueError(f"{op}: A and B must be contiguous")
    if b.ndim != 2 or b_s.ndim != 2:
        raise ValueError(f"{op}: B and Bs must be 2-D")
    k = a.shape[-1]
    m = a.numel() // k
    n, k_b = b.shape
    if k != k_b:
        raise ValueError(f"inner dim mismatch: A K={k}, B K={k_b}")
    n_tiles = math.ceil(n / block_n)
    k_tiles = math.ceil(k / block_k)
    if a_s.shape[:-1] != a.shape[:-1] or a_s.shape[-1] != k_tiles:
        raise ValueError(
            f"{op}: As shape {tuple(a_s.shape)} incompatible "
            f"with A {tuple(a.shape)} and block_k={block_k}"
        )
    if b_s.shape != (n_tiles, k_tiles):
        raise ValueError(f"{op}: Bs shape {tuple(b_s.shape)} expected ({n_tiles}, {k_tiles})")
    return m, n, k


def _run_w8a8(entry, op, a, b, a_s, b_s, block_n, block_k, m, n, k, output_dtype, bias=None,
              acc_out=None):
    _lib.ensure_device(a, op)
    _lib.same_device(op, a, b, a_s, b_s, bias, acc_out)
    oc = _lib.dtype_code(output_dtype, op)
    if output_dtype not in _FLOATS:
        raise TypeError(f"{op}: output_dtype {output_dtype} (float32, float16, bfloat16)")
    a_sf = a_s.to(torch.float32).contiguous()
    b_sf = b_s.to(torch.float32).contiguous()
    c = torch.empty(*a.shape[:-1], n, dtype=output_dtype, device=a.device)
    args = [a.data_ptr(), b.data_ptr(), a_sf.data_ptr(), b_sf.data_ptr(), c.data_ptr(), oc,
            _lib.ptr(bias)]
    if entry == "to_w8a8_i8_gemm":
        args.append(_lib.ptr(acc_out))
    args += [m, n, k, block_n, block_k, _lib.stream_ptr()]
    _lib.call(entry, *args)
    return c


def w8a8_block_int8_matmul(
    a: torch.Tensor,
    b: torch.Tensor,
    a_s: torch.Tensor,
    b_s: torch.Tensor,
    block_size: list[int],
    output_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """W8A8 block matmul ``C = dequant(A) @ dequant(B).T`` (quant_int8.py:180-228), computed
    as exact int32 block sums scaled in fp32."""
    op = "w8a8_block_int8_matmul"
    block_n, block_k = _validate_w8a8(op, a, b, a_s, b_s, block_size)
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise TypeError("w8a8_block_int8_matmul: A and B must be int8")
    m, n, k = _validate_w8a8_rest(op, a, b, a_s, b_s, block_n, block_k)
    return _run_w8a8("to_w8a8_i8_gemm", op, a, b, a_s, b_s, block_n, block_k, m, n, k,
                     output_dtype)


def w8a8_int8_accumulators(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Exact int32 ``A @ B.T`` of int8 operands (the accumulators of
    :func:`w8a8_block_int8_matmul`), exposed so they can be checked bit for bit."""
    op = "w8a8_int8_accumulators"
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise TypeError(f"{op}: A and B must be int8")
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f"{op}: expected A [M, K] and B [N, K]")
    m, k = a.shape
    n = b.shape[0]
    ones_a = torch.ones(m, 1, dtype=torch.float32, device=a.device)
    ones_b = torch.ones(n, 1, dtype=torch.float32, device=a.device)
    acc = torch.empty(m, n, dtype=torch.int32, device=a.device)
    _run_w8a8("to_w8a8_i8_gemm", op, a.contiguous(), b.contiguous(), ones_a, ones_b, 1, k, m, n,
              k, torch.float32, acc_out=acc)
    return acc


def apply_w8a8_block_int8_linear(
    input: torch.Tensor,
    weight: torch.Tensor,
    block_size: list[int],
    weight_scale: torch.Tensor,
    input_scale: Optional[torch.Tensor] = None,
    bias: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Group-quant the input, block W8A8 matmul, add bias (quant_int8.py:231-256). A bias of
    the input's dtype is added inside the GEMM epilogue with the reference's two roundings."""
    if input_scale is not None:
        raise ValueError("apply_w8a8_block_int8_linear: input_scale must be None")
    input_2d = input.view(-1, input.shape[-1])
    output_shape = [*input.shape[:-1], weight.shape[0]]
    q_input, x_scale = per_token_group_quant_int8(input_2d, block_size[1])
    op = "w8a8_block_int8_matmul"
    block_n, block_k = _validate_w8a8(op, q_input, weight, x_scale, weight_scale, block_size)
    if weight.dtype != torch.int8:
        raise TypeError("w8a8_block_int8_matmul: A and B must be int8")
    m, n, k = _validate_w8a8_rest(op, q_input, weight, x_scale, weight_scale, block_n, block_k)
    fuse = bias is not None and bias.dtype == input.dtype and bias.numel() == n
    output = _run_w8a8("to_w8a8_i8_gemm", op, q_input, weight, x_scale, weight_scale, block_n,
                       block_k, m, n, k, input.dtype,
                       bias=bias.contiguous() if fuse else None)
    if bias is not None and not fuse:
        output = output + bias
    return output.to(dtype=input.dtype).view(*output_shape)


__all__ = [
    "apply_w8a8_block_int8_linear",
    "block_dequant",
    "input_to_int8",
    "per_token_group_quant_int8",
    "per_token_quant_int8",
    "w8a8_block_int8_matmul",
]
