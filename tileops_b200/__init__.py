"""tileops_b200: the TileOps quantized-linear hot path, rebuilt for B200 (sm_100a).

Exposes the same names as the reference facade's quant section (tileops/__init__.py:213-248):
AWQ W4A16 pack/unpack/dequant/GEMM, INT8 W8A8 dynamic quantisation and block-scaled
matmul, FP8 e4m3 dynamic quantisation and block-scaled matmul, and symmetric INT8
quantize/dequantize. Every op runs a hand-written CUDA kernel from libtileops_b200.so;
there is no CPU path.
"""

from .quant import (
    dequantize_per_channel,
    dequantize_per_tensor,
    quantize_per_channel,
    quantize_per_tensor,
)
from .quant_awq import (
    AWQ_TRITON_SUPPORTED_GROUP_SIZES,
    REVERSE_AWQ_ORDER,
    awq_dequantize,
    awq_dequantize_triton,
    awq_gemm,
    awq_gemm_gelu_and_mul,
    awq_gemm_silu_and_mul,
    awq_gemm_triton,
    awq_interleave_gate_up,
    pack_awq_int4,
    unpack_awq_int4,
)
from .quant_fp8 import (
    apply_w8a8_block_fp8_linear,
    block_dequant as block_dequant_fp8,
    default_fp8_dtype,
    get_fp8_min_max,
    input_to_float8,
    is_fp8,
    per_token_group_quant_fp8,
    per_token_group_quant_fp8_tma_aligned,
    w8a8_block_fp8_matmul,
    w8a8_triton_block_scaled_mm,
)
from .quant_int8 import (
    apply_w8a8_block_int8_linear,
    block_dequant,
    input_to_int8,
    per_token_group_quant_int8,
    per_token_quant_int8,
    w8a8_block_int8_matmul,
    w8a8_int8_accumulators,
)
from ._lib import set_launch_overlap, version
from .blas import gemm, gemv, mm, mv
from .fused import act_and_mul_group_quant, gelu_and_mul, silu_and_mul

__all__ = [
    "set_launch_overlap",
    "quantize_per_tensor",
    "dequantize_per_tensor",
    "quantize_per_channel",
    "dequantize_per_channel",
    "input_to_int8",
    "input_to_float8",
    "is_fp8",
    "default_fp8_dtype",
    "get_fp8_min_max",
    "per_token_quant_int8",
    "per_token_group_quant_int8",
    "per_token_group_quant_fp8",
    "per_token_group_quant_fp8_tma_aligned",
    "block_dequant",
    "block_dequant_fp8",
    "w8a8_block_int8_matmul",
    "w8a8_block_fp8_matmul",
    "w8a8_triton_block_scaled_mm",
    "w8a8_int8_accumulators",
    "apply_w8a8_block_int8_linear",
    "apply_w8a8_block_fp8_linear",
    "AWQ_TRITON_SUPPORTED_GROUP_SIZES",
    "REVERSE_AWQ_ORDER",
    "awq_dequantize",
    "awq_dequantize_triton",
    "act_and_mul_group_quant",
    "awq_gemm",
    "awq_gemm_gelu_and_mul",
    "awq_gemm_silu_and_mul",
    "awq_gemm_triton",
    "awq_interleave_gate_up",
    "pack_awq_int4",
    "unpack_awq_int4",
    "version",
    "silu_and_mul",
    "gelu_and_mul",
    "gemm",
    "mm",
    "gemv",
    "mv",
]
