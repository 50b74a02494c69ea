"""GPU parity of the gated activations (silu_and_mul, gelu_and_mul): against the golden
vectors (torch CPU ``act(a) * b``, the comparator of the reference's tests/fused.py), the CPU
oracle on strided, ragged and multi-dimensional inputs, and the reference tests' own cases
(out=, a transposed out, validation errors)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import tileops_b200 as tob
from oracle import fused as ofused

pytestmark = pytest.mark.gpu

_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
_OPS = {"silu": tob.silu_and_mul, "gelu": tob.gelu_and_mul}


def _check(got: torch.Tensor, want: np.ndarray, dt: str) -> None:
    g = got.float().cpu().numpy()
    if dt == "f32":
        np.testing.assert_allclose(g, want, rtol=1e-5, atol=1e-6)
    else:  # within two ulps of the 16-bit result (the activation is rounded once before)
        ulp = 2.0 ** (-10 if dt == "f16" else -7)
        np.testing.assert_allclose(g, want, rtol=2 * ulp, atol=1e-6)


@pytest.mark.parametrize("name", [f"{op}{w}_{dt}" for op in ("silu", "gelu")
                                  for w in ("", "_wide") for dt in ("f32", "f16", "bf16")])
def test_golden(cuda, golden, name):
    c = golden("fused.npz")[name]
    y = _OPS[name.split("_")[0]](c.tensor("a", cuda), c.tensor("b", cuda))
    assert y.dtype == c.tensor("a").dtype
    _check(y, np.asarray(c["c"]), c.dtype_name("a"))


@pytest.mark.parametrize("op", ["silu", "gelu"])
@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("shape", [(1,), (1000,), (7, 33), (3, 5, 7), (64, 4096)])
def test_vs_oracle(cuda, op, dt, shape):
    g = torch.Generator().manual_seed(sum(shape) + len(dt))
    a = (torch.randn(*shape, generator=g) * 4).to(_DT[dt])
    b = torch.randn(*shape, generator=g).to(_DT[dt])
    y = _OPS[op](a.to(cuda), b.to(cuda))
    _check(y, ofused.act_and_mul(a.float().numpy(), b.float().numpy(), op, dt), dt)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_gate_up_halves_in_place(cuda, dt):
    """The decode layer's use: the gate and up halves of a [M, 2F] gate_up output, read as
    strided views, into a fresh [M, F] and into a column slice of a wider out."""
    g = torch.Generator().manual_seed(5)
    m, f = 16, 14336
    u = (torch.randn(m, 2 * f, generator=g) * 3).to(_DT[dt])
    uc = u.to(cuda)
    y = tob.silu_and_mul(uc[:, :f], uc[:, f:])
    want = ofused.act_and_mul(u[:, :f].float().numpy(), u[:, f:].float().numpy(), "silu", dt)
    assert y.shape == (m, f) and y.is_contiguous()
    _check(y, want, dt)
    wide = torch.full((m, f + 64), 7.0, dtype=_DT[dt], device=cuda)
    r = tob.silu_and_mul(uc[:, :f], uc[:, f:], out=wide[:, 32:32 + f])
    _check(r, want, dt)
    assert bool((wide[:, :32] == 7).all()) and bool((wide[:, 32 + f:] == 7).all())


def test_reference_cases(cuda):
    """tests/fused.py of the reference, restated: f32 (32, 128) against torch's own ops, the
    out= form returning out itself, and a transposed (non-contiguous) out."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(32, 128, generator=g).to(cuda)
    b = torch.randn(32, 128, generator=g).to(cuda)
    torch.testing.assert_close(tob.silu_and_mul(a, b), F.silu(a) * b, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(tob.gelu_and_mul(a, b), F.gelu(a, approximate="tanh") * b,
                               rtol=1e-2, atol=1e-2)
    o = torch.empty_like(a)
    assert tob.silu_and_mul(a, b, out=o) is o
    torch.testing.assert_close(o, F.silu(a) * b, rtol=1e-2, atol=1e-2)
    a2 = torch.randn(4, 3, generator=g).to(cuda)
    b2 = torch.randn(4, 3, generator=g).to(cuda)
    ot = torch.empty(3, 4, device=cuda).t()
    assert not ot.is_contiguous()
    assert tob.silu_and_mul(a2, b2, out=ot) is ot
    torch.testing.assert_close(ot, F.silu(a2) * b2, rtol=1e-2, atol=1e-2)


def test_validation(cuda):
    a = torch.randn(2, 3, device=cuda)
    with pytest.raises(ValueError):
        tob.silu_and_mul(a, torch.randn(2, 4, device=cuda))
    with pytest.raises(TypeError):
        tob.silu_and_mul(a, a.half())
    with pytest.raises(ValueError):
        tob.gelu_and_mul(a, a, out=torch.empty(3, 2, device=cuda))
    with pytest.raises(TypeError):
        tob.silu_and_mul(a.to(torch.int32), a.to(torch.int32))
    e = torch.empty(0, 5, device=cuda)
    assert tob.silu_and_mul(e, e).shape == (0, 5)


@pytest.mark.parametrize("act", ["silu", "gelu"])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,f,g,opts", [
    (16, 14336, 128, {}),                                 # the decode step's gate_up, FP8
    (7, 512, 64, {"use_ue8m0": True}),
    (33, 1024, 128, {"column_major_scales": True}),
    (5, 768, 128, {"dtype": torch.int8}),
    (300, 96, 32, {}),                                    # odd group size: scalar loads
])
def test_act_and_mul_group_quant_equals_the_two_ops(cuda, act, dt, rows, f, g, opts):
    """The fused activation + per-token-group quantiser against silu_and_mul / gelu_and_mul
    followed by per_token_group_quant_fp8 / _int8, bit for bit, on the gate and up halves of a
    gate_up output read in place; and against the oracle."""
    gen = torch.Generator().manual_seed(rows * 13 + f + g)
    u = (torch.randn(rows, 2 * f, generator=gen) * 3).to(dt).to(cuda)
    u[0, 3] = float("nan")
    gate, up = u[:, :f], u[:, f:]
    q, s = tob.act_and_mul_group_quant(gate, up, g, act=act, **opts)
    y = (tob.silu_and_mul if act == "silu" else tob.gelu_and_mul)(gate, up)
    if opts.get("dtype") == torch.int8:
        wq, ws = tob.per_token_group_quant_int8(y, g)
    else:
        wq, ws = tob.per_token_group_quant_fp8(
            y, g, column_major_scales=opts.get("column_major_scales", False),
            use_ue8m0=opts.get("use_ue8m0", False))
    assert q.dtype == wq.dtype and q.shape == wq.shape and s.shape == ws.shape
    assert torch.equal(q.view(torch.uint8) if q.dtype != torch.int8 else q,
                       wq.view(torch.uint8) if wq.dtype != torch.int8 else wq)
    assert np.array_equal(s.cpu().numpy(), ws.cpu().numpy(), equal_nan=True)
