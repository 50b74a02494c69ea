"""GPU parity of the quantisation kernels against the golden vectors (the reference's own
outputs) and the CPU oracle: bit-exact for every quantised code and scale."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tileops_b200 as tob
from oracle import fp8 as ofp8
from oracle import int8 as oi8
from oracle import numerics
from oracle import sym as osym

pytestmark = pytest.mark.gpu

_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _codes(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e4m3fnuz):
        return t.view(torch.uint8).cpu().numpy()
    return t.cpu().numpy()


def _f(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _same(a, b) -> bool:
    """Equal values, a NaN matching a NaN (scales of groups that hold a NaN)."""
    if isinstance(a, torch.Tensor):
        a = a.float().cpu().numpy()
    return np.array_equal(np.asarray(a, np.float32), np.asarray(b, np.float32), equal_nan=True)


_NAN = ("float32", "float16", "bfloat16")


# ------------------------------------------------------------------ symmetric INT8
@pytest.mark.parametrize("name", ["q_known", "q_ties", "roundtrip", "q_nan"])
def test_quantize_per_tensor_golden(cuda, golden, name):
    c = golden("sym.npz")[name]
    q = tob.quantize_per_tensor(c.tensor("x", cuda), c.tensor("s", cuda))
    assert q.dtype == torch.int8
    assert np.array_equal(q.cpu().numpy(), c["q"])


def test_dequantize_per_tensor_golden(cuda, golden):
    for name in ("dq_known", "roundtrip"):
        c = golden("sym.npz")[name]
        y = tob.dequantize_per_tensor(c.tensor("q", cuda), c.tensor("s", cuda))
        assert np.array_equal(y.cpu().numpy(), c["y"])


@pytest.mark.parametrize("name", ["ch_last", "ch_inner"])
def test_quantize_per_channel_golden(cuda, golden, name):
    c = golden("sym.npz")[name]
    q = tob.quantize_per_channel(c.tensor("x", cuda), c.tensor("s", cuda), dim=int(c["dim"]))
    assert np.array_equal(q.cpu().numpy(), c["q"])


def test_dequantize_per_channel_golden(cuda, golden):
    c = golden("sym.npz")["dq_ch"]
    y = tob.dequantize_per_channel(c.tensor("q", cuda), c.tensor("s", cuda), dim=int(c["dim"]))
    assert np.array_equal(y.cpu().numpy(), c["y"])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("shape,dim", [((1000,), None), ((7, 33, 5), 1), ((64, 129), -1),
                                       ((3, 4, 1031), 0)])
def test_symmetric_random_vs_oracle(cuda, dtype, shape, dim):
    g = torch.Generator().manual_seed(hash((dtype, shape)) & 0xFFFF)
    x = (torch.randn(*shape, generator=g) * 4).to(_DT[dtype])
    if dim is None:
        s = torch.tensor([0.037], dtype=torch.float32)
        q = tob.quantize_per_tensor(x.to(cuda), s.to(cuda))
        want = osym.quantize(_f(x), s.numpy())
        y = tob.dequantize_per_tensor(q, s.to(cuda), out_dtype=_DT[dtype])
        want_y = osym.dequantize(want, s.numpy(), dtype)
    else:
        n = shape[dim]
        s = torch.rand(n, generator=g) * 0.05 + 0.01
        q = tob.quantize_per_channel(x.to(cuda), s.to(cuda), dim)
        want = osym.quantize(_f(x), s.numpy(), dim)
        y = tob.dequantize_per_channel(q, s.to(cuda), dim, out_dtype=_DT[dtype])
        want_y = osym.dequantize(want, s.numpy(), dtype, dim)
    assert np.array_equal(q.cpu().numpy(), want)
    assert np.array_equal(_f(y), want_y)


def test_quantize_out_is_returned(cuda):
    x = torch.randn(10, device=cuda)
    s = torch.tensor([0.2], device=cuda)
    out = torch.empty_like(x, dtype=torch.int8)
    assert tob.quantize_per_tensor(x, s, out=out) is out
    assert np.array_equal(out.cpu().numpy(), osym.quantize(_f(x), s.cpu().numpy()))
    out_nc = torch.empty(20, dtype=torch.int8, device=cuda)[::2]
    assert tob.quantize_per_tensor(x, s, out=out_nc) is out_nc
    assert np.array_equal(out_nc.cpu().numpy(), out.cpu().numpy())


def test_scale_must_be_positive(cuda):
    with pytest.raises(ValueError):
        tob.quantize_per_tensor(torch.randn(4, device=cuda), torch.tensor([0.0], device=cuda))


def test_empty_inputs(cuda):
    s = torch.tensor([0.1], device=cuda)
    assert tob.quantize_per_tensor(torch.empty(0, device=cuda), s).numel() == 0
    q, sc = tob.per_token_quant_int8(torch.empty(0, 16, device=cuda))
    assert q.shape == (0, 16) and sc.shape == (0, 1)


# ------------------------------------------------------------------ dynamic INT8
@pytest.mark.parametrize("name", ["input_known", "input_float32", "input_float16", "input_bfloat16",
                                  "input_zeros_float32", "input_zeros_float16",
                                  "input_zeros_bfloat16", "input_tiny_float16"]
                         + [f"input_nan_{d}" for d in _NAN])
def test_input_to_int8_golden(cuda, golden, name):
    c = golden("int8.npz")[name]
    q, s = tob.input_to_int8(c.tensor("x", cuda))
    assert q.dtype == torch.int8
    assert np.array_equal(q.cpu().numpy(), c["q"])
    assert _same(s, c["s"])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", [1, 7, 4096, 1 << 20, (1 << 20) + 13])
def test_input_to_int8_vs_oracle(cuda, dtype, n):
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(n, generator=g) * 3).to(_DT[dtype])
    q, s = tob.input_to_int8(x.to(cuda))
    wq, ws = oi8.input_to_int8(_f(x), dtype)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert np.float32(s.item()) == ws


@pytest.mark.parametrize("name", ["token_2d", "token_nd", "token_bf16", "token_1d", "token_wide",
                                  "token_edges"] + [f"token_nan_{d}" for d in _NAN])
def test_per_token_quant_int8_golden(cuda, golden, name):
    c = golden("int8.npz")[name]
    q, s = tob.per_token_quant_int8(c.tensor("x", cuda))
    assert q.shape == tuple(c["q"].shape) and s.shape == tuple(c["s"].shape)
    assert np.array_equal(q.cpu().numpy(), c["q"])
    assert _same(s, c["s"])


@pytest.mark.parametrize("name", ["group_f32", "group_bf16", "group_f16_3d", "group_edges"]
                         + [f"group_nan_{d}" for d in _NAN])
def test_per_token_group_quant_int8_golden(cuda, golden, name):
    c = golden("int8.npz")[name]
    q, s = tob.per_token_group_quant_int8(c.tensor("x", cuda), int(c["group_size"]))
    assert np.array_equal(q.cpu().numpy(), c["q"])
    assert _same(s, c["s"])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows,k,g", [(1, 8, 8), (37, 24, 8), (64, 128, 128), (3, 4096, 4096),
                                      (5, 16384, 16384), (2, 65536, 65536), (9, 3000, 1000),
                                      (256, 4096, 128)])
def test_group_quant_int8_vs_oracle(cuda, dtype, rows, k, g):
    gen = torch.Generator().manual_seed(rows * 7 + k)
    x = (torch.randn(rows, k, generator=gen) * 2).to(_DT[dtype])
    q, s = tob.per_token_group_quant_int8(x.to(cuda), g)
    wq, ws = oi8.group_quant(_f(x), g)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert np.array_equal(s.cpu().numpy(), ws)


# ------------------------------------------------------------------ dynamic FP8
@pytest.mark.parametrize("name", ["input_known", "input_float32", "input_float16", "input_bfloat16",
                                  "input_zeros_float32", "input_zeros_float16",
                                  "input_zeros_bfloat16"]
                         + [f"input_{k}_{d}" for k in ("nan", "inf") for d in _NAN])
def test_input_to_float8_golden(cuda, golden, name):
    c = golden("fp8.npz")[name]
    q, s = tob.input_to_float8(c.tensor("x", cuda))
    assert q.dtype == torch.float8_e4m3fn
    assert np.array_equal(_codes(q), c["q"])
    assert _same(s, c["s"])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", [3, 4099, 1 << 21])
def test_input_to_float8_vs_oracle(cuda, dtype, n):
    g = torch.Generator().manual_seed(n + 5)
    x = (torch.randn(n, generator=g) * 7).to(_DT[dtype])
    q, s = tob.input_to_float8(x.to(cuda))
    wq, ws = ofp8.input_to_float8(_f(x), dtype)
    assert np.array_equal(_codes(q), wq)
    assert np.float32(s.item()) == ws


@pytest.mark.parametrize("name", ["group_f32", "group_ue8m0", "group_bf16_token", "group_f16",
                                  "group_colmajor", "group_colmajor_3d", "group_ue8m0_bf16",
                                  "ue8m0_edges"]
                         + [f"group_nan_{d}{u}" for d in _NAN for u in ("", "_ue8m0")]
                         + ["group_zero_eps0"])
def test_per_token_group_quant_fp8_golden(cuda, golden, name):
    c = golden("fp8.npz")[name]
    eps = float(c["eps"]) if "eps" in c else 1e-10
    q, s = tob.per_token_group_quant_fp8(c.tensor("x", cuda), int(c["group_size"]), eps=eps,
                                         column_major_scales=bool(c["column_major"]),
                                         use_ue8m0=bool(c["ue8m0"]))
    assert np.array_equal(_codes(q), c["q"])
    assert s.shape == tuple(c["s"].shape)
    assert _same(s, c["s"])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows,k,g,ue8m0", [(3, 32, 8, False), (128, 512, 128, True),
                                            (64, 8192, 8192, False), (7, 7168, 128, True),
                                            (33, 1536, 96, False)])
def test_group_quant_fp8_vs_oracle(cuda, dtype, rows, k, g, ue8m0):
    gen = torch.Generator().manual_seed(rows + k + g)
    x = (torch.randn(rows, k, generator=gen) * 5).to(_DT[dtype])
    q, s = tob.per_token_group_quant_fp8(x.to(cuda), g, use_ue8m0=ue8m0)
    wq, ws = ofp8.group_quant(_f(x), g, use_ue8m0=ue8m0)
    assert np.array_equal(_codes(q), wq)
    assert np.array_equal(s.cpu().numpy(), ws)


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", [37, 4099, (1 << 20) + 13])
def test_tensor_wide_nan_vs_oracle(cuda, dtype, n):
    """A NaN anywhere makes the tensor's scale NaN: every int8 code 0, every e4m3 code a NaN
    code with the sign the reference's host run gives it."""
    g = torch.Generator().manual_seed(n + 11)
    x = (torch.randn(n, generator=g) * 2).to(_DT[dtype])
    x[torch.randint(0, n, (3,), generator=g)] = float("nan")
    q, s = tob.input_to_float8(x.to(cuda))
    wq, ws = ofp8.input_to_float8(_f(x), dtype)
    assert np.array_equal(_codes(q), wq)
    assert _same(s, ws)
    q, s = tob.input_to_int8(x.to(cuda))
    wq, ws = oi8.input_to_int8(_f(x), dtype)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert _same(s, ws)


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows,k,g", [(37, 24, 8), (64, 8192, 8192), (256, 4096, 128),
                                      (5, 65536, 65536)])
def test_group_nan_inf_vs_oracle(cuda, dtype, rows, k, g):
    """NaN and +-inf inside groups, for every team shape of the group kernel."""
    gen = torch.Generator().manual_seed(rows + k + 3)
    x = (torch.randn(rows, k, generator=gen) * 2).to(_DT[dtype])
    flat = x.view(-1)
    idx = torch.randint(0, flat.numel(), (6,), generator=gen)
    flat[idx[:3]] = float("nan")
    flat[idx[3]] = float("inf")
    flat[idx[4]] = float("-inf")
    for ue8m0 in (False, True):
        q, s = tob.per_token_group_quant_fp8(x.to(cuda), g, use_ue8m0=ue8m0)
        wq, ws = ofp8.group_quant(_f(x), g, use_ue8m0=ue8m0)
        assert np.array_equal(_codes(q), wq)
        assert _same(s, ws)
    q, s = tob.per_token_group_quant_int8(x.to(cuda), g)
    wq, ws = oi8.group_quant(_f(x), g)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert _same(s, ws)


def test_group_quant_fp8_out_q(cuda):
    x = torch.randn(4, 64, device=cuda)
    out = torch.empty(4, 64, dtype=torch.float8_e4m3fn, device=cuda)
    q, s = tob.per_token_group_quant_fp8(x, 16, out_q=out)
    assert q is out
    wq, ws = ofp8.group_quant(_f(x), 16)
    assert np.array_equal(_codes(out), wq)


# ------------------------------------------------------------------ block dequant
def test_block_dequant_int8_golden(cuda, golden):
    c = golden("int8.npz")["block_dequant"]
    y = tob.block_dequant(c.tensor("q", cuda), c.tensor("s", cuda), list(c["block"]))
    assert np.array_equal(y.cpu().numpy(), c["y"])


def test_block_dequant_fp8_golden(cuda, golden):
    c = golden("fp8.npz")["block_dequant"]
    y = tob.block_dequant_fp8(c.tensor("q", cuda), c.tensor("s", cuda), list(c["block"]))
    assert np.array_equal(y.cpu().numpy(), c["y"])


@pytest.mark.parametrize("n,k,bn,bk", [(300, 1000, 128, 128), (129, 257, 1, 257), (64, 64, 64, 64)])
def test_block_dequant_vs_oracle(cuda, n, k, bn, bk):
    g = torch.Generator().manual_seed(n * k)
    q = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8)
    s = torch.rand(-(-n // bn), -(-k // bk), generator=g) * 0.1 + 0.001
    y = tob.block_dequant(q.to(cuda), s.to(cuda), [bn, bk])
    assert np.array_equal(y.cpu().numpy(), oi8.block_dequant(q.numpy(), s.numpy(), (bn, bk)))
    qf = (torch.randn(n, k, generator=g) * 3).clamp(-448, 448).to(torch.float8_e4m3fn)
    y = tob.block_dequant_fp8(qf.to(cuda), s.to(cuda), [bn, bk])
    want = ofp8.block_dequant(qf.view(torch.uint8).numpy(), s.numpy(), (bn, bk))
    assert np.array_equal(y.cpu().numpy(), want)


# ------------------------------------------------------------------ FP8 e4m3fnuz codes
_FNUZ = torch.float8_e4m3fnuz
_FNUZ_DT = ("float32", "float16", "bfloat16")


@pytest.mark.parametrize("name", [f"input_{k}{dt}" for k in ("", "nan_", "zeros_")
                                  for dt in _FNUZ_DT])
def test_input_to_float8_fnuz_golden(cuda, golden, name):
    c = golden("fnuz.npz")[name]
    q, s = tob.input_to_float8(c.tensor("x", cuda), dtype=_FNUZ)
    assert q.dtype == _FNUZ
    assert np.array_equal(_codes(q), c["q"])
    assert _same(s, c["s"])


@pytest.mark.parametrize("name", [f"group_{dt}{u}" for dt in _FNUZ_DT for u in ("", "_ue8m0")]
                         + ["group_colmajor"])
def test_per_token_group_quant_fp8_fnuz_golden(cuda, golden, name):
    c = golden("fnuz.npz")[name]
    q, s = tob.per_token_group_quant_fp8(c.tensor("x", cuda), int(c["group_size"]), dtype=_FNUZ,
                                         column_major_scales=bool(c["column_major"]),
                                         use_ue8m0=bool(c["ue8m0"]))
    assert q.dtype == _FNUZ
    assert np.array_equal(_codes(q), c["q"])
    assert _same(s, c["s"])


def test_block_dequant_fnuz_golden(cuda, golden):
    c = golden("fnuz.npz")["block_dequant"]
    y = tob.block_dequant_fp8(c.tensor("q", cuda), c.tensor("s", cuda),
                              [int(v) for v in c["block"]])
    assert np.array_equal(y.cpu().numpy(), c["y"])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("n", [37, 4099, (1 << 20) + 13])
def test_fnuz_quantisers_vs_oracle(cuda, dtype, n):
    """Both e4m3fnuz quantisers against the oracle, with NaN and inf inside (every NaN code
    0x80), and every code decoded back by block_dequant."""
    g = torch.Generator().manual_seed(n + 17)
    x = (torch.randn(n, generator=g) * 9).to(_DT[dtype])
    x[torch.randint(0, n, (2,), generator=g)] = float("nan")
    x[torch.randint(0, n, (1,), generator=g)] = float("inf")
    q, s = tob.input_to_float8(x.to(cuda), dtype=_FNUZ)
    wq, ws = ofp8.input_to_float8(_f(x), dtype, fnuz=True)
    assert np.array_equal(_codes(q), wq)
    assert _same(s, ws)
    x2 = x[: (n // 16) * 16].view(-1, 16) if n >= 16 else x.view(1, -1)
    g2 = x2.shape[-1]
    for ue8m0 in (False, True):
        q, s = tob.per_token_group_quant_fp8(x2.to(cuda), g2, dtype=_FNUZ, use_ue8m0=ue8m0)
        wq, ws = ofp8.group_quant(_f(x2), g2, use_ue8m0=ue8m0, fnuz=True)
        assert np.array_equal(_codes(q), wq)
        assert _same(s, ws)
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(1, 256)
    y = tob.block_dequant_fp8(codes.view(_FNUZ).to(cuda), torch.ones(1, 1, device=cuda),
                              [1, 256])
    assert _same(y.cpu().numpy().reshape(-1), numerics.e4m3fnuz_to_f32(np.arange(256)))


def test_fnuz_gemm_rejected(cuda):
    a = torch.zeros(4, 16, device=cuda).to(_FNUZ)
    b = torch.zeros(16, 16, device=cuda).to(_FNUZ)
    with pytest.raises(NotImplementedError):
        tob.w8a8_block_fp8_matmul(a, b, torch.ones(4, 1, device=cuda),
                                  torch.ones(1, 1, device=cuda), [16, 16])


@pytest.mark.parametrize("rows,k,g,ue8m0", [(5, 256, 128, False), (33, 7168, 128, True),
                                            (128, 512, 64, False), (1, 128, 128, False)])
def test_group_quant_fp8_tma_aligned_scales(cuda, rows, k, g, ue8m0):
    """The TMA-aligned column-major scale layout: the same codes and scale values as the row
    layout, each group's column of scales 16-byte aligned (leading dimension rows rounded up to
    4)."""
    gen = torch.Generator().manual_seed(rows + k)
    x = (torch.randn(rows, k, generator=gen) * 3).bfloat16().to(cuda)
    q, s = tob.per_token_group_quant_fp8_tma_aligned(x, g, use_ue8m0=ue8m0)
    wq, ws = tob.per_token_group_quant_fp8(x, g, use_ue8m0=ue8m0)
    ld = (rows + 3) // 4 * 4
    assert s.shape == (rows, k // g) and s.stride() == (1, ld)
    assert s.data_ptr() % 16 == 0
    assert torch.equal(q.view(torch.uint8), wq.view(torch.uint8))
    assert torch.equal(s, ws)


def test_symmetric_quant_captures_in_a_graph(cuda):
    """quantize_per_tensor inside a CUDA graph capture: the scale's host-side value check (a
    device read) is skipped while capturing, and replays match eager calls."""
    x = torch.randn(4096, device=cuda)
    s = torch.tensor([0.05], device=cuda)
    want = tob.quantize_per_tensor(x, s)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        tob.quantize_per_tensor(x, s)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = tob.quantize_per_tensor(x, s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    del g


def _midpoint_groups(kind: str) -> np.ndarray:
    """Groups of 16 fp32 values: the group's absmax A first, then 15 values x whose quotient
    x / scale lies on or within four fp32 ulps of a rounding boundary of the code grid: an e4m3
    rounding midpoint (scale A / 448) or a half-integer (int8, scale A / 127)."""
    if kind == "fp8":
        vals = np.unique(np.abs(numerics.E4M3_VALUES[~np.isnan(numerics.E4M3_VALUES)]))
        mids = ((vals[:-1].astype(np.float64) + vals[1:]) / 2).astype(np.float32)
        qmax = np.float32(448.0)
    else:
        mids = (np.arange(0, 127, dtype=np.float32) + np.float32(0.5)).astype(np.float32)
        qmax = np.float32(127.0)
    gen = np.random.default_rng(21)
    groups = []
    for amax in (448.0, 1.0, 3.7, 1e-3, 12345.678, 2.0 ** -20):
        a = np.float32(amax)
        scale = np.float32(a / qmax)
        for k in range(-4, 5):
            x = (mids * scale).astype(np.float32)
            step = np.float32(np.inf) if k > 0 else np.float32(-np.inf)
            for _ in range(abs(k)):
                x = np.nextafter(x, step)
            x = x * np.where(gen.random(x.size) < 0.5, -1.0, 1.0).astype(np.float32)
            x = x[np.abs(x) < a]
            for c in range(0, x.size, 15):
                chunk = x[c:c + 15]
                groups.append(np.concatenate([[a], chunk, np.zeros(15 - chunk.size, np.float32)]))
    return np.stack(groups).astype(np.float32)


@pytest.mark.parametrize("kind", ["fp8", "int8"])
def test_group_quant_quotients_at_rounding_boundaries(cuda, kind):
    """The kernel brackets x / scale between x * lo and x * hi (lo, hi just either side of
    1 / scale) and divides exactly only where the two give different codes: on quotients on
    and around every rounding boundary, across the normal and subnormal e4m3 range and the
    int8 range, its codes must be those of the exact IEEE division (the oracle)."""
    x = _midpoint_groups(kind)
    xt = torch.from_numpy(x).to(cuda)
    if kind == "fp8":
        q, s = tob.per_token_group_quant_fp8(xt, 16)
        wq, ws = ofp8.group_quant(x, 16)
        got = _codes(q)
    else:
        q, s = tob.per_token_group_quant_int8(xt, 16)
        wq, ws = oi8.group_quant(x, 16)
        got = q.cpu().numpy()
    assert np.array_equal(s.cpu().numpy(), ws)
    assert np.array_equal(got, wq)
    # The same values one to a thread (an odd row length leaves the vector path).
    xo = np.concatenate([x, x[:, :1]], axis=1)[:, :17]
    xo_t = torch.from_numpy(np.ascontiguousarray(xo)).to(cuda)
    if kind == "fp8":
        q1, s1 = tob.per_token_group_quant_fp8(xo_t, 17)
        wq1, ws1 = ofp8.group_quant(xo, 17)
        got1 = _codes(q1)
    else:
        q1, s1 = tob.per_token_group_quant_int8(xo_t, 17)
        wq1, ws1 = oi8.group_quant(xo, 17)
        got1 = q1.cpu().numpy()
    assert np.array_equal(s1.cpu().numpy(), ws1)
    assert np.array_equal(got1, wq1)
