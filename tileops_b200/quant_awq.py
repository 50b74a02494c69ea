"""AWQ W4A16 facade: pack/unpack, dequantize and ``x @ dequant(W)`` on sm_100a.

Drop-in for tileops/quant_awq.py: same names, arguments, validation order and messages,
packed layouts (eight int4 per int32 in AWQ nibble order (0,4,1,5,2,6,3,7),
quant_awq.py:19-22) and scale/zero conventions (``(w - z) * s`` per K-group). The math runs
in libtileops_b200: the streaming GEMV for small M and the tcgen05 GEMM for prefill.
"""

from __future__ import annotations

import torch

from . import _lib

# Supported group sizes; -1 is a sentinel and G == K is always accepted (quant_awq.py:19).
AWQ_TRITON_SUPPORTED_GROUP_SIZES = [-1, 32, 64, 128]

# Nibble position of logical column i inside its packed word (quant_awq.py:22).
REVERSE_AWQ_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)


def _infer_group_size(k: int, num_groups: int) -> int:
    """quant_awq.py:25-28."""
    if num_groups <= 0 or k % num_groups != 0:
        raise ValueError(f"invalid AWQ group layout: K={k}, num_groups={num_groups}")
    return k // num_groups


def _validate_group_size(group_size: int, k: int) -> None:
    """quant_awq.py:31-38."""
    if group_size > k:
        raise ValueError(f"group_size {group_size} must be <= K={k}")
    if group_size not in AWQ_TRITON_SUPPORTED_GROUP_SIZES and group_size != k:
        raise ValueError(
            f"group_size {group_size} not in {AWQ_TRITON_SUPPORTED_GROUP_SIZES} "
            f"and not full K={k}"
        )


def unpack_awq_int4(packed: torch.Tensor) -> torch.Tensor:
    """Unpack AWQ words to int64 nibbles in ``[0, 15]``; the last dim grows by 8
    (quant_awq.py:41-52)."""
    op = "unpack_awq_int4"
    if packed.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"unpack_awq_int4: expected int32 packed tensor, got {packed.dtype}")
    _lib.ensure_device(packed, op)
    if packed.ndim == 0:
        raise ValueError(f"{op}: expected at least 1 dimension")
    p = packed.contiguous()
    cols8 = p.shape[-1]
    rows = p.numel() // cols8 if cols8 else 0
    out = torch.empty(*p.shape[:-1], cols8 * 8, dtype=torch.int64, device=p.device)
    _lib.call("to_awq_unpack", p.data_ptr(), _lib.DTYPE_CODES[p.dtype], out.data_ptr(), rows,
              cols8, _lib.stream_ptr())
    return out


def pack_awq_int4(unpacked: torch.Tensor) -> torch.Tensor:
    """Pack nibbles ``[..., cols]`` (``cols % 8 == 0``) into AWQ int32 words
    (quant_awq.py:55-65). Only the low 4 bits of each value are kept; words whose top
    nibble is >= 8 wrap to negative int32 as in the reference."""
    if unpacked.shape[-1] % 8 != 0:
        raise ValueError("pack_awq_int4: last dimension must be divisible by 8")
    op = "pack_awq_int4"
    _lib.ensure_device(unpacked, op)
    u = unpacked
    if u.dtype not in (torch.int32, torch.int64):
        u = u.to(torch.int64)
    u = u.contiguous()
    cols8 = u.shape[-1] // 8
    rows = u.numel() // (cols8 * 8) if cols8 else 0
    out = torch.empty(*u.shape[:-1], cols8, dtype=torch.int32, device=u.device)
    _lib.call("to_awq_pack", u.data_ptr(), _lib.DTYPE_CODES[u.dtype], out.data_ptr(), rows, cols8,
              _lib.stream_ptr())
    return out


def _as_words(t: torch.Tensor) -> torch.Tensor:
    # int64 packed words keep their low 32 bits, as the reference's unpack does.
    if t.dtype == torch.int64:
        t = t.to(torch.int32)
    elif t.dtype != torch.int32:
        raise TypeError(f"unpack_awq_int4: expected int32 packed tensor, got {t.dtype}")
    return t.contiguous()


def awq_dequantize_triton(
    qweight: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    block_size_x: int = 32,
    block_size_y: int = 32,
) -> torch.Tensor:
    """Dequantize AWQ ``qweight [K, N/8]`` with ``scales [K/G, N]`` and ``zeros [K/G, N/8]``
    to ``[K, N]`` in ``scales.dtype`` (quant_awq.py:68-109). ``block_size_*`` are accepted
    for API compatibility."""
    del block_size_x, block_size_y
    op = "awq_dequantize_triton"
    if qweight.ndim != 2 or scales.ndim != 2 or zeros.ndim != 2:
        raise ValueError("awq_dequantize_triton: qweight, scales, zeros must be 2-D")
    k, packed_m = qweight.shape
    m = packed_m * 8
    num_groups = scales.shape[0]
    group_size = _infer_group_size(k, num_groups)
    if k <= 0 or m <= 0:
        raise ValueError(f"awq_dequantize_triton: invalid shape K={k}, M={m}")
    if scales.shape[1] != m:
        raise ValueError(f"awq_dequantize_triton: scales.shape[1]={scales.shape[1]} != M={m}")
    if zeros.shape != (num_groups, packed_m):
        raise ValueError(
            f"awq_dequantize_triton: zeros shape {tuple(zeros.shape)} expected "
            f"({num_groups}, {packed_m})"
        )
    _validate_group_size(group_size, k)
    _lib.ensure_device(qweight, op)
    _lib.same_device(op, qweight, scales, zeros)
    sd = _lib.dtype_code(scales.dtype, op)
    qw = _as_words(qweight)
    qz = _as_words(zeros)
    s = scales.contiguous()
    out = torch.empty(k, m, dtype=scales.dtype, device=qweight.device)
    _lib.call("to_awq_dequant", qw.data_ptr(), s.data_ptr(), sd, qz.data_ptr(), out.data_ptr(),
              k, m, group_size, _lib.stream_ptr())
    return out


def _gemm_args(op: str, input: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
               qzeros: torch.Tensor, split_k_iters: int):
    """The reference's checks of awq_gemm_triton (quant_awq.py:125-151), in its order and with
    its messages; returns (M, K, N, group size)."""
    if input.ndim != 2:
        raise ValueError(f"{op}: input must be 2-D [M, K]")
    m, k = input.shape
    qws = qweight.shape
    if qws[0] != k:
        raise ValueError(f"{op}: qweight rows {qws[0]} != K={k}")
    n = qws[1] * 8
    qzs = qzeros.shape
    num_groups = qzs[0]
    group_size = _infer_group_size(k, num_groups)
    if n <= 0 or m <= 0:
        raise ValueError(f"{op}: invalid M={m}, N={n}, K={k}")
    if qws[1] != n // 8:
        raise ValueError(f"{op}: qweight column count mismatch")
    if qzs[1] != n // 8:
        raise ValueError(f"{op}: qzeros column count mismatch")
    if scales.shape != (num_groups, n):
        raise ValueError(
            f"{op}: scales shape {tuple(scales.shape)} expected "
            f"({num_groups}, {n})"
        )
    if split_k_iters <= 0 or (split_k_iters & (split_k_iters - 1)) != 0:
        raise ValueError(f"{op}: split_k_iters must be a positive power of 2")
    if split_k_iters > 32:
        raise ValueError(f"{op}: split_k_iters must be <= 32")
    _validate_group_size(group_size, k)
    _lib.ensure_device(input, op)
    _lib.same_device(op, input, qweight, scales, qzeros)
    if scales.dtype not in (torch.float16, torch.bfloat16):
        raise NotImplementedError(f"{op}: scales dtype {scales.dtype} (fp16 and bf16 are "
                                  "supported)")
    return m, k, n, group_size


def awq_gemm_triton(
    input: torch.Tensor,
    qweight: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    split_k_iters: int,
    block_size_m: int = 32,
    block_size_n: int = 32,
    block_size_k: int = 32,
) -> torch.Tensor:
    """AWQ GEMM ``input [M, K] @ dequant(qweight) [K, N]`` in ``scales.dtype``
    (quant_awq.py:112-155). ``split_k_iters`` is validated as in the reference and does not
    change the result; the kernel picks its own K split."""
    del block_size_m, block_size_n, block_size_k
    m, k, n, group_size = _gemm_args("awq_gemm_triton", input, qweight, scales, qzeros,
                                     split_k_iters)
    out_dtype = scales.dtype
    qw = _as_words(qweight)
    qz = _as_words(qzeros)
    s = scales.contiguous()
    dev = input.get_device()
    y = torch.empty(m, n, dtype=out_dtype, device=dev)
    lib = _lib.load()
    st = _lib.stream_ptr(dev)
    ws_bytes = _lib.workspace_bytes("to_awq_gemm_workspace_size", m, k, n, group_size)
    ws = _lib.workspace(ws_bytes, dev, st)
    same_dtype = input.dtype == out_dtype
    contiguous = input.is_contiguous()
    if (same_dtype and not contiguous and input.stride(1) == 1
            and input.stride(0) >= k and input.stride(0) % 8 == 0
            and input.data_ptr() % 16 == 0):
        # a row-strided slice (the first K columns of a wider activation): read in place where
        # the kernel takes a row stride
        rc = lib.to_awq_gemm_strided(input.data_ptr(), input.stride(0), qw.data_ptr(),
                                     s.data_ptr(), _lib.DTYPE_CODES[out_dtype], qz.data_ptr(),
                                     y.data_ptr(), m, k, n, group_size, _lib.ptr(ws), ws_bytes,
                                     st)
        if rc != _lib.TO_EUNSUPPORTED:
            _lib.check(rc, "awq_gemm_triton")
            return y
    x = input if same_dtype and contiguous else input.to(out_dtype).contiguous()
    _lib.call("to_awq_gemm", x.data_ptr(), qw.data_ptr(), s.data_ptr(),
              _lib.DTYPE_CODES[out_dtype], qz.data_ptr(), y.data_ptr(), m, k, n, group_size,
              _lib.ptr(ws), ws_bytes, st)
    return y


# ---------------------------------------------------------------- library extensions
# The gate_up linear of an MLP block with its gated activation in the GEMM (no reference
# counterpart: the reference runs awq_gemm, then tileops/fused.py:97 silu_and_mul on the two
# halves of its output).

ACT_SILU = 0
ACT_GELU_TANH = 1


def awq_interleave_gate_up(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor):
    """The weight layout awq_gemm_silu_and_mul / awq_gemm_gelu_and_mul read, from a gate_up
    linear whose N columns hold gate in [0, N/2) and up in [N/2, N): gate and up alternate in
    blocks of 8 columns (one packed word): block 2j = gate columns 8j..8j+7, block 2j + 1 = up
    columns 8j..8j+7. A one-time reordering of whole words and scale columns (CPU or CUDA
    tensors); returns contiguous (qweight, scales, qzeros)."""
    n = qweight.shape[1] * 8
    if n % 16 != 0:
        raise ValueError(f"awq_interleave_gate_up: N={n} is not a multiple of 16")
    if scales.shape[-1] != n or qzeros.shape[-1] != n // 8:
        raise ValueError("awq_interleave_gate_up: scales / qzeros do not match qweight's N")

    def words(t: torch.Tensor) -> torch.Tensor:
        r = t.shape[0]
        return t.reshape(r, 2, n // 16).transpose(1, 2).reshape(r, n // 8).contiguous()

    g = scales.shape[0]
    s = scales.reshape(g, 2, n // 16, 8).transpose(1, 2).reshape(g, n).contiguous()
    return words(qweight), s, words(qzeros)


def _gemm_act(op: str, act: int, input, qweight, scales, qzeros, split_k_iters) -> torch.Tensor:
    m, k, n, group_size = _gemm_args(op, input, qweight, scales, qzeros, split_k_iters)
    if n % 16 != 0:
        raise ValueError(f"{op}: N={n} is not a multiple of 16 (gate and up blocks of 8)")
    out_dtype = scales.dtype
    x = input if input.dtype == out_dtype and input.is_contiguous() else \
        input.to(out_dtype).contiguous()
    qw = _as_words(qweight)
    qz = _as_words(qzeros)
    s = scales.contiguous()
    dev = input.get_device()
    y = torch.empty(m, n // 2, dtype=out_dtype, device=dev)
    st = _lib.stream_ptr(dev)
    ws_bytes = _lib.workspace_bytes("to_awq_gemm_act_workspace_size", m, k, n, group_size)
    ws = _lib.workspace(ws_bytes, dev, st)
    _lib.call("to_awq_gemm_act", x.data_ptr(), qw.data_ptr(), s.data_ptr(),
              _lib.DTYPE_CODES[out_dtype], qz.data_ptr(), y.data_ptr(), m, k, n, group_size,
              act, _lib.ptr(ws), ws_bytes, st)
    return y


def awq_gemm_silu_and_mul(input: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                          qzeros: torch.Tensor, split_k_iters: int = 1) -> torch.Tensor:
    """``silu(gate) * up`` of the gate_up linear ``input @ dequant(W)``, W interleaved by
    awq_interleave_gate_up: [M, N/2], equal to awq_gemm on the original weights followed by
    silu_and_mul(y[:, :N/2], y[:, N/2:]). Arguments and checks as awq_gemm_triton."""
    return _gemm_act("awq_gemm_silu_and_mul", ACT_SILU, input, qweight, scales, qzeros,
                     split_k_iters)


def awq_gemm_gelu_and_mul(input: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                          qzeros: torch.Tensor, split_k_iters: int = 1) -> torch.Tensor:
    """``gelu_tanh(gate) * up`` of the gate_up linear, as awq_gemm_silu_and_mul."""
    return _gemm_act("awq_gemm_gelu_and_mul", ACT_GELU_TANH, input, qweight, scales, qzeros,
                     split_k_iters)


# vLLM names kept as primary entry points (quant_awq.py:159-160).
awq_dequantize = awq_dequantize_triton
awq_gemm = awq_gemm_triton

__all__ = [
    "AWQ_TRITON_SUPPORTED_GROUP_SIZES",
    "REVERSE_AWQ_ORDER",
    "awq_dequantize",
    "awq_dequantize_triton",
    "awq_gemm",
    "awq_gemm_gelu_and_mul",
    "awq_gemm_silu_and_mul",
    "awq_gemm_triton",
    "awq_interleave_gate_up",
    "pack_awq_int4",
    "unpack_awq_int4",
]
