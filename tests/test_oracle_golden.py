"""Pins the CPU oracle against golden vectors produced by running the reference itself
(tests/golden/make_golden.py) and against the reference tests' known-answer vectors.
Runs without a GPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import awq, fp8, fused, int8, numerics, sym


def _np(case, field):
    return np.asarray(case[field])


# ------------------------------------------------------------------ numerics
def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    vals = numerics.e4m3_to_f32(codes)
    finite = ~np.isnan(vals)
    back = numerics.f32_to_e4m3(vals[finite])
    # +0 and -0 both decode to 0 with their sign; every finite code survives the round trip
    assert np.array_equal(back, codes[finite])


def test_e4m3_round_half_even_midpoints():
    vals = numerics.E4M3_VALUES[:0x7F]
    pos = np.sort(vals[~np.isnan(vals)])
    mids = ((pos[:-1].astype(np.float64) + pos[1:]) / 2).astype(np.float32)
    codes = numerics.f32_to_e4m3(mids)
    lo = numerics.f32_to_e4m3(pos[:-1])
    hi = numerics.f32_to_e4m3(pos[1:])
    # each midpoint goes to whichever neighbour has an even mantissa
    want = np.where((lo & 1) == 0, lo, hi)
    assert np.array_equal(codes, want)


def test_bf16_rounding_matches_torch():
    import torch

    g = np.random.default_rng(0)
    x = (g.standard_normal(10000) * 10.0 ** g.integers(-5, 5, 10000)).astype(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(numerics.round_bf16(x), want)


def test_e4m3_matches_torch_cast():
    import torch

    g = np.random.default_rng(1)
    x = np.clip(g.standard_normal(20000).astype(np.float32) * 50, -448, 448)
    x = np.concatenate([x, numerics.E4M3_VALUES[:0x7F] * 1.0000001, [2.0 ** -10, 3 * 2.0 ** -11]]).astype(np.float32)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(numerics.f32_to_e4m3(x), want)


# ------------------------------------------------------------------ AWQ
def test_awq_pack_unpack(golden):
    g = golden("awq.npz")
    c = g["roundtrip"]
    assert np.array_equal(awq.pack(_np(c, "x")), _np(c, "packed"))
    assert np.array_equal(awq.unpack(_np(c, "packed")), _np(c, "unpacked"))
    c = g["pack_wide"]
    assert np.array_equal(awq.pack(_np(c, "x")), _np(c, "packed"))


@pytest.mark.parametrize("name", ["dequant_f16", "dequant_fullk", "dequant_bf16", "dequant_f32"])
def test_awq_dequant(golden, name):
    c = golden("awq.npz")[name]
    out = awq.dequant(_np(c, "qweight"), _np(c, "scales"), _np(c, "qzeros"), c.dtype_name("scales"))
    assert np.array_equal(out, _np(c, "out"))


@pytest.mark.parametrize("name", ["gemm_f16", "gemm_f16_m1", "gemm_f16_m3", "gemm_bf16",
                                  "gemm_bf16_m1", "gemm_f16_fullk"])
def test_awq_gemm(golden, name):
    c = golden("awq.npz")[name]
    y = awq.gemm(_np(c, "x"), _np(c, "qweight"), _np(c, "scales"), _np(c, "qzeros"),
                 c.dtype_name("scales"))
    np.testing.assert_allclose(y, _np(c, "y"), rtol=1e-2, atol=1e-2)


def test_awq_split_k_invariance(golden):
    c = golden("awq.npz")["gemm_splitk"]
    assert np.array_equal(_np(c, "y1"), _np(c, "y4"))


# ------------------------------------------------------------------ INT8
_NAN_INPUTS = ["input_nan_float32", "input_nan_float16", "input_nan_bfloat16"]
_NAN_TOKENS = ["token_nan_float32", "token_nan_float16", "token_nan_bfloat16"]
_NAN_GROUPS = ["group_nan_float32", "group_nan_float16", "group_nan_bfloat16"]


def _same(a, b) -> bool:
    """Equal values, a NaN matching a NaN (scales of groups that hold a NaN)."""
    return np.array_equal(np.asarray(a, np.float32), np.asarray(b, np.float32), equal_nan=True)


@pytest.mark.parametrize("name", ["input_known", "input_float32", "input_float16", "input_bfloat16",
                                  "input_zeros_float32", "input_zeros_float16",
                                  "input_zeros_bfloat16", "input_tiny_float16"] + _NAN_INPUTS)
def test_input_to_int8(golden, name):
    c = golden("int8.npz")[name]
    q, s = int8.input_to_int8(_np(c, "x"), c.dtype_name("x"))
    assert np.array_equal(q, _np(c, "q"))
    assert _same(s, _np(c, "s"))


@pytest.mark.parametrize("name", ["token_2d", "token_nd", "token_bf16", "token_1d", "token_wide",
                                  "token_edges"] + _NAN_TOKENS)
def test_per_token_quant_int8(golden, name):
    c = golden("int8.npz")[name]
    x = _np(c, "x")
    q, s = int8.group_quant(x.reshape(-1, x.shape[-1]), x.shape[-1])
    assert np.array_equal(q.reshape(x.shape), _np(c, "q"))
    assert _same(s.reshape(-1), _np(c, "s").reshape(-1))


@pytest.mark.parametrize("name", ["group_f32", "group_bf16", "group_f16_3d", "group_edges"]
                         + _NAN_GROUPS)
def test_group_quant_int8(golden, name):
    c = golden("int8.npz")[name]
    q, s = int8.group_quant(_np(c, "x"), int(c["group_size"]))
    assert np.array_equal(q, _np(c, "q"))
    assert _same(s, _np(c, "s"))


def test_block_dequant_int8(golden):
    c = golden("int8.npz")["block_dequant"]
    y = int8.block_dequant(_np(c, "q"), _np(c, "s"), list(_np(c, "block")))
    assert np.array_equal(y, _np(c, "y"))


def test_w8a8_int8(golden):
    c = golden("int8.npz")["w8a8_small"]
    y = int8.block_matmul(_np(c, "a"), _np(c, "b"), _np(c, "a_s"), _np(c, "b_s"),
                          list(_np(c, "block")), "f32")
    np.testing.assert_allclose(y, _np(c, "c"), rtol=1e-4, atol=1e-4)
    c = golden("int8.npz")["w8a8_channel"]
    assert np.array_equal(int8.accumulators(_np(c, "a"), _np(c, "b")), _np(c, "acc"))
    y = int8.block_matmul(_np(c, "a"), _np(c, "b"), _np(c, "a_s"), _np(c, "b_s"),
                          list(_np(c, "block")), "bf16")
    np.testing.assert_allclose(y, _np(c, "c"), rtol=1e-2, atol=1e-2)


def test_w8a8_reference_cpu_port_matches(golden):
    c = golden("int8.npz")["w8a8_channel"]
    y = int8.block_matmul_reference_cpu(_np(c, "a"), _np(c, "b"), _np(c, "a_s"), _np(c, "b_s"),
                                        list(_np(c, "block")), "bf16")
    np.testing.assert_allclose(y, _np(c, "c"), rtol=1e-2, atol=1e-2)


# ------------------------------------------------------------------ FP8
_FP8_NAN_INPUTS = [f"input_{k}_{dt}" for k in ("nan", "inf")
                   for dt in ("float32", "float16", "bfloat16")]
_FP8_NAN_GROUPS = [f"group_nan_{dt}{u}" for dt in ("float32", "float16", "bfloat16")
                   for u in ("", "_ue8m0")] + ["group_zero_eps0"]


@pytest.mark.parametrize("name", ["input_known", "input_float32", "input_float16", "input_bfloat16",
                                  "input_zeros_float32", "input_zeros_float16",
                                  "input_zeros_bfloat16"] + _FP8_NAN_INPUTS)
def test_input_to_float8(golden, name):
    c = golden("fp8.npz")[name]
    q, s = fp8.input_to_float8(_np(c, "x"), c.dtype_name("x"))
    assert np.array_equal(q, _np(c, "q"))
    assert _same(s, _np(c, "s"))


@pytest.mark.parametrize("name", ["group_f32", "group_ue8m0", "group_bf16_token", "group_f16",
                                  "group_colmajor", "group_colmajor_3d", "group_ue8m0_bf16",
                                  "ue8m0_edges"] + _FP8_NAN_GROUPS)
def test_group_quant_fp8(golden, name):
    c = golden("fp8.npz")[name]
    eps = float(c["eps"]) if "eps" in c else 1e-10
    q, s = fp8.group_quant(_np(c, "x"), int(c["group_size"]), eps=eps, use_ue8m0=bool(c["ue8m0"]),
                           column_major=bool(c["column_major"]))
    assert np.array_equal(q, _np(c, "q"))
    assert _same(s, _np(c, "s"))


def test_block_dequant_fp8(golden):
    c = golden("fp8.npz")["block_dequant"]
    y = fp8.block_dequant(_np(c, "q"), _np(c, "s"), list(_np(c, "block")))
    assert np.array_equal(y, _np(c, "y"))


_FNUZ_DT = ("float32", "float16", "bfloat16")


@pytest.mark.parametrize("name", [f"input_{k}{dt}" for k in ("", "nan_", "zeros_")
                                  for dt in _FNUZ_DT])
def test_input_to_float8_fnuz(golden, name):
    c = golden("fnuz.npz")[name]
    q, s = fp8.input_to_float8(_np(c, "x"), c.dtype_name("x"), fnuz=True)
    assert np.array_equal(q, _np(c, "q"))
    assert _same(s, _np(c, "s"))


@pytest.mark.parametrize("name", [f"group_{dt}{u}" for dt in _FNUZ_DT for u in ("", "_ue8m0")]
                         + ["group_colmajor"])
def test_group_quant_fp8_fnuz(golden, name):
    c = golden("fnuz.npz")[name]
    q, s = fp8.group_quant(_np(c, "x"), int(c["group_size"]), use_ue8m0=bool(c["ue8m0"]),
                           column_major=bool(c["column_major"]), fnuz=True)
    assert np.array_equal(q, _np(c, "q"))
    assert _same(s, _np(c, "s"))


def test_block_dequant_fp8_fnuz(golden):
    c = golden("fnuz.npz")["block_dequant"]
    y = fp8.block_dequant(_np(c, "q"), _np(c, "s"), list(_np(c, "block")), fnuz=True)
    assert np.array_equal(y, _np(c, "y"))


def test_fnuz_encoding_matches_torch():
    """The oracle's e4m3fnuz rounding against torch's CPU cast (the reference's conversion),
    over ties, subnormals, zero signs and the top of the range."""
    g = torch.Generator().manual_seed(7)
    x = torch.cat([torch.randn(50000, generator=g) * 40, torch.randn(20000, generator=g) * 1e-3,
                   torch.linspace(-240, 240, 48001),
                   torch.tensor([0.0, -0.0, 232.0, -232.0, 2.0 ** -11, -2.0 ** -11])])
    x = x.clamp(-240, 240)
    want = x.to(torch.float8_e4m3fnuz).view(torch.uint8).numpy()
    assert np.array_equal(numerics.f32_to_e4m3fnuz(x.numpy()), want)
    codes = np.arange(256, dtype=np.uint8)
    back = torch.from_numpy(codes).view(torch.float8_e4m3fnuz).float().numpy()
    assert _same(numerics.e4m3fnuz_to_f32(codes), back)


def test_w8a8_fp8(golden):
    c = golden("fp8.npz")["w8a8_small"]
    y = fp8.block_matmul(_np(c, "a"), _np(c, "b"), _np(c, "a_s"), _np(c, "b_s"),
                         list(_np(c, "block")), "f32")
    np.testing.assert_allclose(y, _np(c, "c"), rtol=1e-4, atol=1e-4)


def test_fp8_layer(golden):
    c = golden("fp8.npz")["fp8_layer"]
    A, B = _np(c, "A"), _np(c, "B")
    qa, sa = fp8.group_quant(A, A.shape[1])
    assert np.array_equal(qa, _np(c, "qa")) and np.array_equal(sa, _np(c, "sa"))
    qb, sb = fp8.input_to_float8(B, "bf16")
    assert np.array_equal(qb, _np(c, "qb")) and np.float32(sb) == np.float32(_np(c, "sb"))
    y = fp8.block_matmul(qa, qb, sa, np.array([[sb]], np.float32), [B.shape[0], A.shape[1]], "bf16")
    np.testing.assert_allclose(y, _np(c, "c"), rtol=1e-2, atol=1e-2)


# ------------------------------------------------------------------ symmetric INT8
@pytest.mark.parametrize("name", ["q_known", "q_ties", "roundtrip", "q_zero_scale", "q_nan"])
def test_sym_quant_per_tensor(golden, name):
    c = golden("sym.npz")[name]
    assert np.array_equal(sym.quantize(_np(c, "x"), _np(c, "s")), _np(c, "q"))


def test_sym_dequant(golden):
    g = golden("sym.npz")
    c = g["dq_known"]
    assert np.array_equal(sym.dequantize(_np(c, "q"), _np(c, "s"), "f32"), _np(c, "y"))
    c = g["roundtrip"]
    assert np.array_equal(sym.dequantize(_np(c, "q"), _np(c, "s"), "f32"), _np(c, "y"))
    c = g["dq_ch"]
    assert np.array_equal(sym.dequantize(_np(c, "q"), _np(c, "s"), "f32", int(c["dim"])), _np(c, "y"))


@pytest.mark.parametrize("name", ["ch_last", "ch_inner", "ch_zero_scale"])
def test_sym_quant_per_channel(golden, name):
    c = golden("sym.npz")[name]
    assert np.array_equal(sym.quantize(_np(c, "x"), _np(c, "s"), int(c["dim"])), _np(c, "q"))


# ------------------------------------------------------------------ gated activations
_FUSED = [f"{op}{w}_{dt}" for op in ("silu", "gelu") for w in ("", "_wide")
          for dt in ("f32", "f16", "bf16")]


@pytest.mark.parametrize("name", _FUSED)
def test_fused_act_and_mul_vs_golden(golden, name):
    """The oracle against torch CPU ``act(a) * b``, the comparator of the reference's tests:
    fp32 within rounding of the exp/tanh implementations; 16-bit outputs within two ulps (torch
    may round the 16-bit activation one ulp apart from the correctly rounded fp32 value)."""
    c = golden("fused.npz")[name]
    dt = c.dtype_name("a")
    got = fused.act_and_mul(_np(c, "a"), _np(c, "b"), name.split("_")[0], dt)
    want = _np(c, "c")
    if dt == "f32":
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    else:
        ulp = 2.0 ** (-10 if dt == "f16" else -7)
        np.testing.assert_allclose(got, want, rtol=2 * ulp, atol=1e-6)
