"""Invalid calls shared by make_errors.py (run against the reference) and tests/test_abi.py (run
against this library): each raises during argument checking, before any device work, so both
sides run them on CPU tensors. input_to_int8 with a non-int8 dtype is left out on purpose: the
reference computes it, this library raises NotImplementedError."""

from __future__ import annotations

import torch


def cases(qa, q8, qf, qs, fz) -> dict:
    """qa, q8, qf, qs, fz: the quant_awq, quant_int8, quant_fp8, quant and fused modules."""
    f16, i32, i8 = torch.float16, torch.int32, torch.int8
    z = torch.zeros
    e4m3 = torch.float8_e4m3fn
    return {
        "awq_unpack_bad_dtype": lambda: qa.unpack_awq_int4(z(4, 2)),
        "awq_pack_bad_cols": lambda: qa.pack_awq_int4(z(4, 7, dtype=i32)),
        "awq_dequant_extra_arg": lambda: qa.awq_dequantize(
            z(64, 2, dtype=i32), z(1, 16, dtype=f16), z(1, 2, dtype=i32), 0, 0, 0),
        "awq_gemm_bad_split": lambda: qa.awq_gemm(
            z(2, 64, dtype=f16), z(64, 2, dtype=i32), z(1, 16, dtype=f16), z(1, 2, dtype=i32), 48),
        "awq_gemm_k_mismatch": lambda: qa.awq_gemm(
            z(2, 32, dtype=f16), z(64, 2, dtype=i32), z(1, 16, dtype=f16), z(1, 2, dtype=i32), 64),
        "i8_group_indivisible": lambda: q8.per_token_group_quant_int8(z(2, 10), 4),
        "i8_block_dequant_short_block": lambda: q8.block_dequant(z(4, 8, dtype=i8), z(1, 1), [4]),
        "i8_w8a8_short_block": lambda: q8.w8a8_block_int8_matmul(
            z(2, 8, dtype=i8), z(4, 8, dtype=i8), z(2, 1), z(1, 1), [4]),
        "fp8_group_indivisible": lambda: qf.per_token_group_quant_fp8(z(2, 10), 4),
        "fp8_group_bad_dtype": lambda: qf.per_token_group_quant_fp8(z(2, 8), 4, dtype=torch.int8),
        "fp8_group_tma": lambda: qf.per_token_group_quant_fp8(z(2, 8), 4, tma_aligned_scales=True),
        "fp8_block_dequant_short_block": lambda: qf.block_dequant(z(4, 8).to(e4m3), z(1, 1), [4]),
        "sym_scale_dtype": lambda: qs.quantize_per_tensor(z(4), z(1, dtype=f16)),
        "sym_scale_numel": lambda: qs.quantize_per_tensor(z(4), z(2)),
        "sym_scale_nonpositive": lambda: qs.quantize_per_tensor(z(4), z(1)),
        "sym_channel_bad_dim": lambda: qs.quantize_per_channel(z(4, 3), torch.ones(3), dim=5),
        "sym_int_input": lambda: qs.quantize_per_tensor(z(4, dtype=i32), torch.ones(1)),
        "fused_shape": lambda: fz.silu_and_mul(z(2, 3), z(2, 4)),
        "fused_dtype": lambda: fz.gelu_and_mul(z(2, 3), z(2, 3, dtype=f16)),
    }


def run(table: dict) -> dict:
    """name -> [exception type name, message] (["", ""] if nothing was raised)."""
    out = {}
    for name, fn in table.items():
        try:
            fn()
            out[name] = ["", ""]
        except Exception as e:  # noqa: BLE001 -- the exception itself is the result
            out[name] = [type(e).__name__, str(e)]
    return out
