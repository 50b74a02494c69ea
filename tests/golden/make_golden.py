"""Generates the golden fixtures in this folder by running the REFERENCE implementation
(llongmarch/TileOps, imported from the checkout named by the required TILEOPS_REF variable)
on seeded CPU inputs.

    TILEOPS_REF=<path to a TileOps checkout> python tests/golden/make_golden.py

Writes awq.npz, int8.npz, fp8.npz, fnuz.npz, sym.npz, fused.npz (or only the files named on the
command line: awq, int8, fp8, fnuz, sym, fused). Each case stores its inputs and the reference's
outputs; float tensors are stored as float32 values (bf16/fp16 values are exact in fp32)
with the source dtype under "<case>/<field>.dtype", FP8 tensors as uint8 codes. The
symmetric-INT8 ops have no CPU path in the reference (its TileLang kernels need a GPU
target), so their goldens come from the restatements in the reference's own
tests/quant.py (_ref_* functions), which pin those ops' semantics.

This script is the only code in the repository that imports the reference; nothing that
runs on the GPU box does.
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if not os.environ.get("TILEOPS_REF"):
    sys.exit("set TILEOPS_REF to the TileOps checkout whose outputs the goldens record")
REF = Path(os.environ["TILEOPS_REF"])
sys.path.insert(0, str(REF))

import torch  # noqa: E402

import tileops  # noqa: E402  (the reference package)
import tileops.quant_awq as awq  # noqa: E402
import tileops.quant_fp8 as fp8  # noqa: E402
import tileops.quant_int8 as i8  # noqa: E402

assert Path(tileops.__file__).resolve().is_relative_to(REF.resolve()), tileops.__file__

FP8 = torch.float8_e4m3fn
FNUZ = torch.float8_e4m3fnuz


class Cases:
    def __init__(self):
        self.arrays: dict[str, np.ndarray] = {}

    def put(self, case: str, field: str, t) -> None:
        key = f"{case}/{field}"
        if isinstance(t, torch.Tensor):
            dt = str(t.dtype).replace("torch.", "")
            if t.dtype in (FP8, FNUZ):
                arr = t.contiguous().view(torch.uint8).numpy().copy()
            elif t.dtype in (torch.bfloat16, torch.float16):
                arr = t.float().numpy().copy()
            else:
                arr = t.numpy().copy()
            self.arrays[key] = arr
            self.arrays[key + ".dtype"] = np.array(dt)
        else:
            self.arrays[key] = np.asarray(t)

    def save(self, name: str) -> None:
        np.savez_compressed(HERE / name, **self.arrays)
        print(f"{name}: {len({k.split('/')[0] for k in self.arrays})} cases")


def seed(i: int) -> None:
    torch.manual_seed(1234 + i)


# ------------------------------------------------------------------ AWQ
def make_awq() -> None:
    c = Cases()

    def weights(k, n, g, dtype, lo=0.002, hi=0.02):
        w = torch.randint(0, 16, (k, n), dtype=torch.int64)
        z = torch.randint(0, 16, (k // g, n), dtype=torch.int64)
        s = (torch.rand(k // g, n) * (hi - lo) + lo).to(dtype)
        return awq.pack_awq_int4(w), s, awq.pack_awq_int4(z), w, z

    seed(0)
    x = torch.randint(0, 16, (4, 16), dtype=torch.int64)
    c.put("roundtrip", "x", x)
    c.put("roundtrip", "packed", awq.pack_awq_int4(x))
    c.put("roundtrip", "unpacked", awq.unpack_awq_int4(awq.pack_awq_int4(x)))
    x = torch.randint(0, 16, (8, 64), dtype=torch.int64)
    c.put("pack_wide", "x", x)
    c.put("pack_wide", "packed", awq.pack_awq_int4(x))

    for i, (name, k, n, g, dt) in enumerate([
        ("dequant_f16", 64, 128, 32, torch.float16),
        ("dequant_fullk", 32, 64, 32, torch.float16),
        ("dequant_bf16", 256, 64, 128, torch.bfloat16),
        ("dequant_f32", 128, 64, 64, torch.float32),
    ]):
        seed(10 + i)
        qw, s, qz, _, _ = weights(k, n, g, dt, 0.01, 0.11)
        c.put(name, "qweight", qw)
        c.put(name, "scales", s)
        c.put(name, "qzeros", qz)
        c.put(name, "out", awq.awq_dequantize_triton(qw, s, qz))

    for i, (name, m, k, n, g, dt) in enumerate([
        ("gemm_f16", 8, 64, 128, 32, torch.float16),
        ("gemm_f16_m1", 1, 512, 256, 128, torch.float16),
        ("gemm_f16_m3", 3, 256, 384, 64, torch.float16),
        ("gemm_bf16", 4, 256, 128, 64, torch.bfloat16),
        ("gemm_bf16_m1", 1, 1024, 512, 128, torch.bfloat16),
        ("gemm_f16_fullk", 2, 96, 64, 96, torch.float16),
    ]):
        seed(20 + i)
        qw, s, qz, _, _ = weights(k, n, g, dt)
        xx = torch.randn(m, k).to(dt)
        c.put(name, "x", xx)
        c.put(name, "qweight", qw)
        c.put(name, "scales", s)
        c.put(name, "qzeros", qz)
        c.put(name, "y", awq.awq_gemm_triton(xx, qw, s, qz, split_k_iters=1))
    seed(30)
    qw, s, qz, _, _ = weights(32, 64, 32, torch.float16)
    xx = torch.randn(4, 32, dtype=torch.float16)
    c.put("gemm_splitk", "x", xx)
    c.put("gemm_splitk", "qweight", qw)
    c.put("gemm_splitk", "scales", s)
    c.put("gemm_splitk", "qzeros", qz)
    c.put("gemm_splitk", "y1", awq.awq_gemm_triton(xx, qw, s, qz, split_k_iters=1))
    c.put("gemm_splitk", "y4", awq.awq_gemm_triton(xx, qw, s, qz, split_k_iters=4))
    c.save("awq.npz")


# ------------------------------------------------------------------ INT8
def make_int8() -> None:
    c = Cases()
    x = torch.tensor([-1.5, 0.0, 0.5, 2.0], dtype=torch.float32)
    q, s = i8.input_to_int8(x)
    c.put("input_known", "x", x)
    c.put("input_known", "q", q)
    c.put("input_known", "s", s)
    for i, dt in enumerate([torch.float32, torch.float16, torch.bfloat16]):
        seed(40 + i)
        x = (torch.randn(3000) * 2.5).to(dt)
        q, s = i8.input_to_int8(x)
        name = f"input_{str(dt).replace('torch.', '')}"
        c.put(name, "x", x)
        c.put(name, "q", q)
        c.put(name, "s", s)

    # Degenerate tensors: all zeros, and float16 values too small for float16's 1e-12 clamp
    # (1e-12 rounds to 0 in float16, so the reference divides by a zero amax: scale inf,
    # x * scale NaN, which its int8 cast turns into 0 and the dequant scale into 0).
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        x = torch.zeros(40, dtype=dt)
        q, s = i8.input_to_int8(x)
        name = f"input_zeros_{str(dt).replace('torch.', '')}"
        c.put(name, "x", x)
        c.put(name, "q", q)
        c.put(name, "s", s)
    x = torch.tensor([1e-9, -2e-9, 0.0, 3e-8], dtype=torch.float32).to(torch.float16)
    q, s = i8.input_to_int8(x)
    c.put("input_tiny_float16", "x", x)
    c.put("input_tiny_float16", "q", q)
    c.put("input_tiny_float16", "s", s)

    for i, (name, shape, dt, scale) in enumerate([
        ("token_2d", (4, 16), torch.float32, 0.5),
        ("token_nd", (2, 3, 8), torch.float16, 1.0),
        ("token_bf16", (5, 64), torch.bfloat16, 3.0),
        ("token_1d", (40,), torch.float32, 1.0),
        ("token_wide", (3, 4096), torch.float16, 1.0),
    ]):
        seed(50 + i)
        x = (torch.randn(*shape) * scale).to(dt)
        q, s = i8.per_token_quant_int8(x)
        c.put(name, "x", x)
        c.put(name, "q", q)
        c.put(name, "s", s)

    for i, (name, shape, g, dt) in enumerate([
        ("group_f32", (3, 32), 8, torch.float32),
        ("group_bf16", (4, 256), 128, torch.bfloat16),
        ("group_f16_3d", (2, 2, 96), 24, torch.float16),
    ]):
        seed(60 + i)
        x = torch.randn(*shape).to(dt)
        q, s = i8.per_token_group_quant_int8(x, g)
        c.put(name, "x", x)
        c.put(name, "group_size", np.array(g))
        c.put(name, "q", q)
        c.put(name, "s", s)

    # Zero rows and groups (scale = eps / 127) and exact round-half-even ties (absmax 127
    # makes the scale exactly 1, so x / scale = x).
    x = torch.tensor([[127.0, 0.5, 1.5, 2.5, -0.5, -2.5, 63.5, -126.5],
                      [0.0] * 8,
                      [0.0, 0.0, 0.0, 0.0, 1e-12, -3e-11, 0.0, 0.0]], dtype=torch.float32)
    q, s = i8.per_token_quant_int8(x)
    c.put("token_edges", "x", x)
    c.put("token_edges", "q", q)
    c.put("token_edges", "s", s)
    q, s = i8.per_token_group_quant_int8(x, 4)
    c.put("group_edges", "x", x)
    c.put("group_edges", "group_size", np.array(4))
    c.put("group_edges", "q", q)
    c.put("group_edges", "s", s)

    # NaN and inf inputs. torch's amax / aminmax propagate NaN: the group's (or tensor's) scale
    # is NaN and every code of it 0 (the int8 cast of NaN); an inf makes the scale inf.
    for i, dt in enumerate((torch.float32, torch.float16, torch.bfloat16)):
        tag = str(dt).replace("torch.", "")
        seed(74 + i)
        x = torch.randn(100).to(dt)
        x[5] = float("nan")
        q, s = i8.input_to_int8(x)
        c.put(f"input_nan_{tag}", "x", x)
        c.put(f"input_nan_{tag}", "q", q)
        c.put(f"input_nan_{tag}", "s", s)
        x = torch.randn(4, 64).to(dt)
        x[2, 17] = float("nan")
        q, s = i8.per_token_quant_int8(x)
        c.put(f"token_nan_{tag}", "x", x)
        c.put(f"token_nan_{tag}", "q", q)
        c.put(f"token_nan_{tag}", "s", s)
        x = torch.randn(3, 64).to(dt)
        x[0, 3] = float("nan")
        x[1, 40] = float("inf")
        x[2, 63] = float("-inf")
        q, s = i8.per_token_group_quant_int8(x, 16)
        c.put(f"group_nan_{tag}", "x", x)
        c.put(f"group_nan_{tag}", "group_size", np.array(16))
        c.put(f"group_nan_{tag}", "q", q)
        c.put(f"group_nan_{tag}", "s", s)

    seed(70)
    bs = [4, 8]
    wq = torch.randint(-128, 127, (10, 24), dtype=torch.int8)
    ws = torch.rand(3, 3) * 0.1 + 0.01
    c.put("block_dequant", "q", wq)
    c.put("block_dequant", "s", ws)
    c.put("block_dequant", "block", np.array(bs))
    c.put("block_dequant", "y", i8.block_dequant(wq, ws, bs))

    # w8a8 6x10x24, block [4, 8], constructed as the reference's test does
    seed(71)
    m, n, k = 6, 10, 24
    a = torch.randn(m, k)
    b = torch.randn(n, k)
    q_a, s_a = i8.per_token_group_quant_int8(a, 8)
    q_b = torch.clamp(torch.round(b / 0.05), -128, 127).to(torch.int8)
    s_b = torch.empty(3, 3)
    for j in range(3):
        for ii in range(3):
            blk = q_b[j * 4:min((j + 1) * 4, n), ii * 8:min((ii + 1) * 8, k)].float()
            s_b[j, ii] = blk.abs().max().clamp(min=1e-10) / 127.0
    c.put("w8a8_small", "a", q_a)
    c.put("w8a8_small", "b", q_b)
    c.put("w8a8_small", "a_s", s_a)
    c.put("w8a8_small", "b_s", s_b)
    c.put("w8a8_small", "block", np.array(bs))
    c.put("w8a8_small", "c", i8.w8a8_block_int8_matmul(q_a, q_b, s_a, s_b, bs, output_dtype=torch.float32))

    # per-token x per-channel (block [1, K]) -> bf16, the layout of the M=256 K=4096 N=11008 layer
    seed(72)
    m, n, k = 16, 64, 256
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), dtype=torch.int8)
    a_s = torch.rand(m, 1) * 0.045 + 0.005
    b_s = torch.rand(n, 1) * 0.009 + 0.001
    c.put("w8a8_channel", "a", a)
    c.put("w8a8_channel", "b", b)
    c.put("w8a8_channel", "a_s", a_s)
    c.put("w8a8_channel", "b_s", b_s)
    c.put("w8a8_channel", "block", np.array([1, k]))
    c.put("w8a8_channel", "c", i8.w8a8_block_int8_matmul(a, b, a_s, b_s, [1, k], output_dtype=torch.bfloat16))
    c.put("w8a8_channel", "acc", (a.double() @ b.double().T).to(torch.int64))

    seed(73)
    x = torch.randn(3, 24, dtype=torch.float16)
    w = torch.randn(10, 24)
    w_q = torch.clamp(torch.round(w / 0.04), -128, 127).to(torch.int8)
    s_w = torch.empty(3, 3)
    for j in range(3):
        for ii in range(3):
            blk = w_q[j * 4:min((j + 1) * 4, 10), ii * 8:min((ii + 1) * 8, 24)].float()
            s_w[j, ii] = blk.abs().max().clamp(min=1e-10) / 127.0
    bias = torch.randn(10, dtype=torch.float16)
    c.put("apply_linear", "x", x)
    c.put("apply_linear", "w", w_q)
    c.put("apply_linear", "w_s", s_w)
    c.put("apply_linear", "bias", bias)
    c.put("apply_linear", "block", np.array(bs))
    c.put("apply_linear", "y", i8.apply_w8a8_block_int8_linear(x, w_q, bs, s_w, bias=bias))
    c.save("int8.npz")


# ------------------------------------------------------------------ FP8
def make_fp8() -> None:
    c = Cases()
    x = torch.tensor([-1.5, 0.0, 0.5, 2.0], dtype=torch.float32)
    q, s = fp8.input_to_float8(x, dtype=FP8)
    c.put("input_known", "x", x)
    c.put("input_known", "q", q)
    c.put("input_known", "s", s)
    for i, dt in enumerate([torch.float32, torch.float16, torch.bfloat16]):
        seed(80 + i)
        x = (torch.randn(4000) * 3.0).to(dt)
        q, s = fp8.input_to_float8(x)
        name = f"input_{str(dt).replace('torch.', '')}"
        c.put(name, "x", x)
        c.put(name, "q", q)
        c.put(name, "s", s)

    for dt in (torch.float32, torch.float16, torch.bfloat16):
        x = torch.zeros(40, dtype=dt)
        q, s = fp8.input_to_float8(x, dtype=FP8)
        name = f"input_zeros_{str(dt).replace('torch.', '')}"
        c.put(name, "x", x)
        c.put(name, "q", q)
        c.put(name, "s", s)

    for i, (name, shape, g, dt, ue, cm) in enumerate([
        ("group_f32", (3, 32), 8, torch.float32, False, False),
        ("group_ue8m0", (2, 16), 8, torch.float32, True, False),
        ("group_bf16_token", (8, 512), 512, torch.bfloat16, False, False),
        ("group_f16", (6, 256), 128, torch.float16, False, False),
        ("group_colmajor", (4, 32), 8, torch.float32, False, True),
        ("group_colmajor_3d", (2, 3, 16), 8, torch.float32, False, True),
        ("group_ue8m0_bf16", (5, 384), 128, torch.bfloat16, True, False),
    ]):
        seed(90 + i)
        x = torch.randn(*shape).to(dt)
        q, s = fp8.per_token_group_quant_fp8(x, g, column_major_scales=cm, use_ue8m0=ue)
        c.put(name, "x", x)
        c.put(name, "group_size", np.array(g))
        c.put(name, "ue8m0", np.array(ue))
        c.put(name, "column_major", np.array(cm))
        c.put(name, "q", q)
        c.put(name, "s", s)

    # UE8M0 near powers of two: group absmax = 448 * 2^e * (1 + d) for tiny d
    rows = []
    for e in (-12, -7, -3, 0, 2, 5):
        for d in (0.0, 2.0 ** -23, 2.0 ** -22, 2.0 ** -20, 2.0 ** -16):
            v = torch.zeros(8)
            v[3] = 448.0 * (2.0 ** e) * (1.0 + d)
            v[5] = -0.3 * (2.0 ** e)
            rows.append(v)
    rows.append(torch.zeros(8))  # a zero group: scale = eps / 448 (rounded up to 2^-42)
    x = torch.stack(rows).to(torch.float32)
    q, s = fp8.per_token_group_quant_fp8(x, 8, use_ue8m0=True)
    c.put("ue8m0_edges", "x", x)
    c.put("ue8m0_edges", "group_size", np.array(8))
    c.put("ue8m0_edges", "ue8m0", np.array(True))
    c.put("ue8m0_edges", "column_major", np.array(False))
    c.put("ue8m0_edges", "q", q)
    c.put("ue8m0_edges", "s", s)

    # NaN and inf inputs. A NaN makes the tensor's / group's scale NaN; the NaN codes carry the
    # sign the reference's x86 run gives them (0x7F or 0xFF). 100 elements = three whole
    # 32-element blocks and a tail of 4, where bfloat16's vectorised and scalar roundings
    # differ. A sign-set NaN input is written through the bit pattern (float16, float32).
    neg_nan = torch.tensor([0xFFC00000], dtype=torch.int64).to(torch.int32).view(torch.float32)
    for i, dt in enumerate((torch.float32, torch.float16, torch.bfloat16)):
        tag = str(dt).replace("torch.", "")
        seed(104 + i)
        x = torch.randn(100).to(dt)
        x[5] = float("nan")
        x[98] = float("nan")
        q, s = fp8.input_to_float8(x, dtype=FP8)
        c.put(f"input_nan_{tag}", "x", x)
        c.put(f"input_nan_{tag}", "q", q)
        c.put(f"input_nan_{tag}", "s", s)
        x = torch.randn(100).to(dt)
        x[2] = float("-inf")
        x[97] = float("inf")
        q, s = fp8.input_to_float8(x, dtype=FP8)
        c.put(f"input_inf_{tag}", "x", x)
        c.put(f"input_inf_{tag}", "q", q)
        c.put(f"input_inf_{tag}", "s", s)
        x = torch.randn(4, 64).to(dt)
        x[0, 3] = float("nan")
        if dt != torch.bfloat16:
            x[1, 20] = neg_nan.to(dt)[0]
        x[2, 40] = float("inf")
        x[3, 63] = float("-inf")
        for ue in (False, True):
            q, s = fp8.per_token_group_quant_fp8(x, 16, dtype=FP8, use_ue8m0=ue)
            name = f"group_nan_{tag}" + ("_ue8m0" if ue else "")
            c.put(name, "x", x)
            c.put(name, "group_size", np.array(16))
            c.put(name, "ue8m0", np.array(ue))
            c.put(name, "column_major", np.array(False))
            c.put(name, "q", q)
            c.put(name, "s", s)
    # a zero group with eps = 0: scale 0, every quotient 0 / 0
    x = torch.zeros(2, 16)
    x[1, :] = torch.randn(16)
    q, s = fp8.per_token_group_quant_fp8(x, 16, eps=0.0, dtype=FP8)
    c.put("group_zero_eps0", "x", x)
    c.put("group_zero_eps0", "group_size", np.array(16))
    c.put("group_zero_eps0", "eps", np.array(0.0))
    c.put("group_zero_eps0", "ue8m0", np.array(False))
    c.put("group_zero_eps0", "column_major", np.array(False))
    c.put("group_zero_eps0", "q", q)
    c.put("group_zero_eps0", "s", s)

    seed(100)
    bs = [4, 8]
    wq = torch.randn(10, 24).clamp(-1, 1).to(FP8)
    ws = torch.rand(3, 3) * 0.1 + 0.01
    c.put("block_dequant", "q", wq)
    c.put("block_dequant", "s", ws)
    c.put("block_dequant", "block", np.array(bs))
    c.put("block_dequant", "y", fp8.block_dequant(wq, ws, bs))

    seed(101)
    m, n, k = 6, 10, 24
    a = torch.randn(m, k)
    b = torch.randn(n, k)
    q_a, s_a = fp8.per_token_group_quant_fp8(a, 8)
    q_b = b.clamp(-1, 1).to(FP8)
    s_b = torch.empty(3, 3)
    for j in range(3):
        for ii in range(3):
            blk = q_b[j * 4:min((j + 1) * 4, n), ii * 8:min((ii + 1) * 8, k)].float()
            s_b[j, ii] = blk.abs().max().clamp(min=1e-10) / 448.0
    c.put("w8a8_small", "a", q_a)
    c.put("w8a8_small", "b", q_b)
    c.put("w8a8_small", "a_s", s_a)
    c.put("w8a8_small", "b_s", s_b)
    c.put("w8a8_small", "block", np.array(bs))
    c.put("w8a8_small", "c", fp8.w8a8_block_fp8_matmul(q_a, q_b, s_a, s_b, bs, output_dtype=torch.float32))

    # the dynamic-quant + per-token x per-tensor GEMM of the M=N=K=8192 layer, scaled down
    seed(102)
    m, n, k = 64, 128, 256
    A = torch.randn(m, k, dtype=torch.bfloat16)
    B = torch.randn(n, k, dtype=torch.bfloat16)
    qa, sa = fp8.per_token_group_quant_fp8(A, k)
    qb, sb = fp8.input_to_float8(B)
    c.put("fp8_layer", "A", A)
    c.put("fp8_layer", "B", B)
    c.put("fp8_layer", "qa", qa)
    c.put("fp8_layer", "sa", sa)
    c.put("fp8_layer", "qb", qb)
    c.put("fp8_layer", "sb", sb)
    c.put("fp8_layer", "c", fp8.w8a8_block_fp8_matmul(qa, qb, sa, sb.reshape(1, 1), [n, k],
                                                       output_dtype=torch.bfloat16))

    seed(103)
    x = torch.randn(3, 24, dtype=torch.float16)
    w_q = torch.randn(10, 24).clamp(-1, 1).to(FP8)
    s_w = torch.empty(3, 3)
    for j in range(3):
        for ii in range(3):
            blk = w_q[j * 4:min((j + 1) * 4, 10), ii * 8:min((ii + 1) * 8, 24)].float()
            s_w[j, ii] = blk.abs().max().clamp(min=1e-10) / 448.0
    bias = torch.randn(10, dtype=torch.float16)
    c.put("apply_linear", "x", x)
    c.put("apply_linear", "w", w_q)
    c.put("apply_linear", "w_s", s_w)
    c.put("apply_linear", "bias", bias)
    c.put("apply_linear", "block", np.array(bs))
    c.put("apply_linear", "y", fp8.apply_w8a8_block_fp8_linear(x, w_q, bs, s_w, bias=bias))
    c.save("fp8.npz")


# ------------------------------------------------------------------ symmetric INT8
def make_sym() -> None:
    spec = importlib.util.spec_from_file_location("ref_tests_quant", REF / "tests" / "quant.py")
    rt = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rt)
    c = Cases()
    x = torch.tensor([-0.25, 0.0, 0.19, 1.05], dtype=torch.float32)
    s = torch.tensor([0.1], dtype=torch.float32)
    c.put("q_known", "x", x)
    c.put("q_known", "s", s)
    c.put("q_known", "q", rt._ref_quantize_per_tensor(x, s))
    qk = torch.tensor([-3, 0, 2, 10], dtype=torch.int8)
    s = torch.tensor([0.05], dtype=torch.float32)
    c.put("dq_known", "q", qk)
    c.put("dq_known", "s", s)
    c.put("dq_known", "y", rt._ref_dequantize_per_tensor(qk, s, torch.float32))
    # exact half-way points: x / s = +-0.5, 1.5, 2.5, ... must round half to even
    x = torch.tensor([0.25, 0.75, 1.25, -0.25, -0.75, 63.75, -64.25, 100.0], dtype=torch.float32)
    s = torch.tensor([0.5], dtype=torch.float32)
    c.put("q_ties", "x", x)
    c.put("q_ties", "s", s)
    c.put("q_ties", "q", rt._ref_quantize_per_tensor(x, s))
    # NaN inputs: round and clamp keep NaN, the int8 cast makes it 0
    x = torch.tensor([float("nan"), 1.0, -0.3, float("nan"), 100.0], dtype=torch.float32)
    s = torch.tensor([0.5], dtype=torch.float32)
    c.put("q_nan", "x", x)
    c.put("q_nan", "s", s)
    c.put("q_nan", "q", rt._ref_quantize_per_tensor(x, s))
    # a zero scale (the public functions reject it; this pins the kernel expression): x / 0 is
    # +-inf (clamped) or, for x = +-0, NaN (int8 cast: 0)
    x = torch.tensor([0.0, 1.0, -2.0, -0.0, 3.5e-3, -1e30], dtype=torch.float32)
    s = torch.tensor([0.0], dtype=torch.float32)
    c.put("q_zero_scale", "x", x)
    c.put("q_zero_scale", "s", s)
    c.put("q_zero_scale", "q", rt._ref_quantize_per_tensor(x, s))
    seed(110)
    x = torch.randn(32, 64) * 0.3
    s = torch.tensor([x.abs().max().item() / 127.0 + 1e-6])
    q = rt._ref_quantize_per_tensor(x, s)
    c.put("roundtrip", "x", x)
    c.put("roundtrip", "s", s)
    c.put("roundtrip", "q", q)
    c.put("roundtrip", "y", rt._ref_dequantize_per_tensor(q, s, torch.float32))
    seed(111)
    x = torch.randn(4, 8)
    s = torch.linspace(0.05, 0.2, 8)
    c.put("ch_last", "x", x)
    c.put("ch_last", "s", s)
    c.put("ch_last", "dim", np.array(-1))
    c.put("ch_last", "q", rt._ref_quantize_per_channel(x, s, -1))
    seed(112)
    x = torch.randn(3, 5, 7)
    s = torch.linspace(0.1, 0.3, 5)
    c.put("ch_inner", "x", x)
    c.put("ch_inner", "s", s)
    c.put("ch_inner", "dim", np.array(1))
    c.put("ch_inner", "q", rt._ref_quantize_per_channel(x, s, 1))
    # one channel with a zero scale, zeros included
    x = torch.tensor([[0.0, 0.3, -0.0], [1.0, -0.5, 0.0], [-2.0, 0.0, 0.25]], dtype=torch.float32)
    s = torch.tensor([0.1, 0.0, 0.05], dtype=torch.float32)
    c.put("ch_zero_scale", "x", x)
    c.put("ch_zero_scale", "s", s)
    c.put("ch_zero_scale", "dim", np.array(-1))
    c.put("ch_zero_scale", "q", rt._ref_quantize_per_channel(x, s, -1))
    seed(113)
    s = torch.tensor([0.1, 0.2, 0.15])
    x = torch.randn(2, 3)
    q = rt._ref_quantize_per_channel(x, s, -1)
    c.put("dq_ch", "q", q)
    c.put("dq_ch", "s", s)
    c.put("dq_ch", "dim", np.array(-1))
    c.put("dq_ch", "y", rt._ref_dequantize_per_channel(q, s, -1, torch.float32))
    c.save("sym.npz")


# ------------------------------------------------------------------ gated activations
def make_fused() -> None:
    """silu_and_mul / gelu_and_mul (tileops/fused.py:97-114) have no CPU path in the reference
    (TileLang kernels), so their goldens are the comparators of the reference's own
    tests/fused.py: ``F.silu(a) * b`` and ``F.gelu(a, approximate="tanh") * b`` on torch CPU,
    here also in fp16 and bf16."""
    import torch.nn.functional as F

    c = Cases()
    for i, (dt, tag) in enumerate(((torch.float32, "f32"), (torch.float16, "f16"),
                                   (torch.bfloat16, "bf16"))):
        seed(120 + i)
        a = torch.randn(32, 128).to(dt)  # the reference test's shape
        b = torch.randn(32, 128).to(dt)
        c.put(f"silu_{tag}", "a", a)
        c.put(f"silu_{tag}", "b", b)
        c.put(f"silu_{tag}", "c", F.silu(a) * b)
        c.put(f"gelu_{tag}", "a", a)
        c.put(f"gelu_{tag}", "b", b)
        c.put(f"gelu_{tag}", "c", F.gelu(a, approximate="tanh") * b)
        # wide range and an odd width: saturated sigmoid, tanh and exp(-x) overflow
        a = (torch.randn(7, 33) * 30).to(dt)
        b = torch.randn(7, 33).to(dt)
        c.put(f"silu_wide_{tag}", "a", a)
        c.put(f"silu_wide_{tag}", "b", b)
        c.put(f"silu_wide_{tag}", "c", F.silu(a) * b)
        c.put(f"gelu_wide_{tag}", "a", a)
        c.put(f"gelu_wide_{tag}", "b", b)
        c.put(f"gelu_wide_{tag}", "c", F.gelu(a, approximate="tanh") * b)
    c.save("fused.npz")


# ------------------------------------------------------------------ FP8 e4m3fnuz
def make_fnuz() -> None:
    """The FP8 quantisers with dtype=torch.float8_e4m3fnuz: tensor-wide to +-240 (finfo), per
    group to get_fp8_min_max's +-224, every NaN code 0x80; block_dequant of fnuz codes."""
    c = Cases()
    for i, dt in enumerate((torch.float32, torch.float16, torch.bfloat16)):
        tag = str(dt).replace("torch.", "")
        seed(300 + i)
        x = (torch.randn(4000) * 3.0).to(dt)
        q, s = fp8.input_to_float8(x, dtype=FNUZ)
        c.put(f"input_{tag}", "x", x)
        c.put(f"input_{tag}", "q", q)
        c.put(f"input_{tag}", "s", s)
        x = torch.randn(100).to(dt)
        x[5] = float("nan")
        q, s = fp8.input_to_float8(x, dtype=FNUZ)
        c.put(f"input_nan_{tag}", "x", x)
        c.put(f"input_nan_{tag}", "q", q)
        c.put(f"input_nan_{tag}", "s", s)
        x = torch.zeros(40, dtype=dt)
        q, s = fp8.input_to_float8(x, dtype=FNUZ)
        c.put(f"input_zeros_{tag}", "x", x)
        c.put(f"input_zeros_{tag}", "q", q)
        c.put(f"input_zeros_{tag}", "s", s)
        for ue in (False, True):
            seed(310 + i)
            x = torch.randn(6, 256).to(dt)
            x[2, 7] = float("nan")
            x[4, 100] = float("inf")
            x[5, :] = 0.0
            q, s = fp8.per_token_group_quant_fp8(x, 64, dtype=FNUZ, use_ue8m0=ue)
            name = f"group_{tag}" + ("_ue8m0" if ue else "")
            c.put(name, "x", x)
            c.put(name, "group_size", np.array(64))
            c.put(name, "ue8m0", np.array(ue))
            c.put(name, "column_major", np.array(False))
            c.put(name, "q", q)
            c.put(name, "s", s)
    seed(320)
    x = torch.randn(4, 32)
    q, s = fp8.per_token_group_quant_fp8(x, 8, dtype=FNUZ, column_major_scales=True)
    c.put("group_colmajor", "x", x)
    c.put("group_colmajor", "group_size", np.array(8))
    c.put("group_colmajor", "ue8m0", np.array(False))
    c.put("group_colmajor", "column_major", np.array(True))
    c.put("group_colmajor", "q", q)
    c.put("group_colmajor", "s", s)
    seed(321)
    bs = [4, 8]
    wq = (torch.randn(10, 24) * 60).clamp(-240, 240).to(FNUZ)
    ws = torch.rand(3, 3) * 0.1 + 0.01
    c.put("block_dequant", "q", wq)
    c.put("block_dequant", "s", ws)
    c.put("block_dequant", "block", np.array(bs))
    c.put("block_dequant", "y", fp8.block_dequant(wq, ws, bs))
    c.save("fnuz.npz")


if __name__ == "__main__":
    torch.set_num_threads(1)
    makers = {"awq": make_awq, "int8": make_int8, "fp8": make_fp8, "fnuz": make_fnuz,
              "sym": make_sym, "fused": make_fused}
    for name in sys.argv[1:] or list(makers):
        makers[name]()
