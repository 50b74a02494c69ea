"""GPU parity of the dense GEMM and GEMV (tileops.gemm / mm, tileops.gemv / mv): the tcgen05
tiles with B read MN-major and the streaming GEMV against an fp32 (fp64 for GEMV) torch product of
the same inputs (rtol = atol = 1e-2 on 16-bit outputs of unit scale, 1e-4 on fp32 GEMV), ragged
shapes, out= and the SIMT tiles for the GEMM shapes and dtypes outside the tcgen05 tiles."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tileops_b200 as tob

pytestmark = pytest.mark.gpu


def _inputs(m, n, k, dt, seed):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) / k ** 0.5).to(dt)
    b = torch.randn(k, n, generator=g).to(dt)
    return a, b


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(256, 512, 1024), (1000, 768, 4000), (64, 1024, 256),
                                   (129, 320, 72), (2048, 2048, 2048),
                                   (4096, 4096, 264),     # 256-row tiles (they fill the SMs)
                                   (4000, 4160, 1000)])   # 256-row tiles, ragged M and K
def test_gemm_vs_fp32(cuda, dt, m, n, k):
    a, b = _inputs(m, n, k, dt, m + n + k)
    c = tob.gemm(a.to(cuda), b.to(cuda))
    assert c.dtype == dt and c.shape == (m, n)
    want = (a.float() @ b.float()).numpy()
    np.testing.assert_allclose(c.float().cpu().numpy(), want, rtol=1e-2, atol=1e-2)


def test_gemm_deterministic_and_out(cuda):
    a, b = _inputs(512, 1024, 2048, torch.bfloat16, 3)
    a, b = a.to(cuda), b.to(cuda)
    c1 = tob.gemm(a, b)
    o = torch.empty(512, 1024, dtype=torch.bfloat16, device=cuda)
    assert tob.mm(a, b, out=o) is o
    assert torch.equal(c1, o)
    ot = torch.empty(1024, 512, dtype=torch.bfloat16, device=cuda).t()
    assert tob.gemm(a, b, out=ot) is ot
    assert torch.equal(ot, c1)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(33, 50, 20), (1, 1, 1), (130, 70, 1001), (300, 200, 64),
                                   (64, 64, 7)])
def test_gemm_simt_tiles_vs_fp64(cuda, dt, m, n, k):
    """Shapes outside the tcgen05 tiles (N % 64, K % 8) and fp32 run on the SIMT tiles."""
    a, b = _inputs(m, n, k, dt, m * 3 + n + k)
    c = tob.gemm(a.to(cuda), b.to(cuda))
    assert c.dtype == dt and c.shape == (m, n)
    want = (a.double() @ b.double()).numpy()
    tol = 1e-5 if dt == torch.float32 else 1e-2
    np.testing.assert_allclose(c.double().cpu().numpy(), want, rtol=tol, atol=tol)


def test_gemm_other_shapes_and_errors(cuda):
    a, b = _inputs(33, 64, 24, torch.float16, 4)
    # an unaligned view of B (offset by one element) leaves the tensor-core tiles too
    bb = torch.empty(24 * 64 + 1, dtype=torch.float16, device=cuda)[1:].view(24, 64)
    bb.copy_(b.to(cuda))
    c = tob.gemm(a.to(cuda), bb)
    np.testing.assert_allclose(c.float().cpu().numpy(), (a.float() @ b.float()).numpy(),
                               rtol=1e-2, atol=1e-2)
    with pytest.raises(ValueError):
        tob.gemm(torch.zeros(2, 3, device=cuda, dtype=torch.int32),
                 torch.zeros(3, 5, device=cuda, dtype=torch.int32))
    with pytest.raises(ValueError):
        tob.gemm(torch.zeros(2, 3, device=cuda), torch.zeros(4, 5, device=cuda))
    with pytest.raises(TypeError):
        tob.gemm(torch.zeros(2, 3, device=cuda), torch.zeros(3, 5, device=cuda).half())
    with pytest.raises(ValueError):
        tob.gemm(torch.zeros(3, device=cuda), torch.zeros(3, 5, device=cuda))


# ---------------------------------------------------------------- GEMV (tileops.gemv / mv)

def _gemv_inputs(m, k, dt, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(dt)
    x = (torch.randn(k, generator=g) / max(k, 1) ** 0.5).to(dt)
    return a, x


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k", [(9, 4), (1, 1), (28672, 512),     # one warp per row
                                 (7, 65536), (300, 8192),    # rows split over 8 / 2 warps
                                 (1000, 33), (513, 1001),    # K not a multiple of the vector
                                 (4096, 4096), (1500, 3000),  # bulk-copy stream, one chunk
                                 (1200, 20000)])             # bulk-copy stream, ragged chunks
def test_gemv_vs_fp32(cuda, dt, m, k):
    a, x = _gemv_inputs(m, k, dt, m * 31 + k)
    y = tob.gemv(a.to(cuda), x.to(cuda))
    assert y.dtype == dt and y.shape == (m,)
    want = (a.double() @ x.double()).numpy()
    tol = 1e-4 if dt == torch.float32 else 1e-2
    np.testing.assert_allclose(y.double().cpu().numpy(), want, rtol=tol, atol=tol)


def test_gemv_reference_cases(cuda):
    # the cases of the reference's dense tests (tests/blas.py:50-75, 158-163), rtol = atol = 1e-3
    g = torch.Generator().manual_seed(0)
    a = torch.randn(9, 4, generator=g).to(cuda)
    x = torch.randn(4, generator=g).to(cuda)
    torch.testing.assert_close(tob.gemv(a, x), a @ x, rtol=1e-3, atol=1e-3)
    a2 = torch.randn(4, 3, generator=g).to(cuda)
    x2 = torch.randn(3, generator=g).to(cuda)
    torch.testing.assert_close(tob.mv(a2, x2), tob.gemv(a2, x2), rtol=1e-3, atol=1e-3)
    a3 = torch.randn(5, 2, generator=g).to(cuda)
    x3 = torch.randn(2, generator=g).to(cuda)
    out = torch.empty(5, device=cuda)
    assert tob.gemv(a3, x3, out=out) is out
    torch.testing.assert_close(out, a3 @ x3, rtol=1e-3, atol=1e-3)
    with pytest.raises(ValueError):
        tob.gemv(torch.randn(3, 4, device=cuda), torch.randn(3, device=cuda))


def test_gemv_layouts_deterministic_and_empty(cuda):
    a, x = _gemv_inputs(2048, 4096, torch.bfloat16, 5)
    a, x = a.to(cuda), x.to(cuda)
    y1 = tob.gemv(a, x)
    assert torch.equal(y1, tob.gemv(a, x))
    # strided out, misaligned x (scalar-load path), transposed A (made contiguous)
    o = torch.zeros(4096, dtype=torch.bfloat16, device=cuda)[::2]
    assert tob.gemv(a, x, out=o) is o and torch.equal(o, y1)
    xb = torch.empty(4097, dtype=torch.bfloat16, device=cuda)
    xb[1:] = x
    y2 = tob.gemv(a, xb[1:])
    np.testing.assert_allclose(y2.float().cpu().numpy(), y1.float().cpu().numpy(), rtol=1e-2,
                               atol=1e-2)
    at = a.t().contiguous().t()
    assert torch.equal(tob.gemv(at, x), y1)
    # K = 0 gives zeros, M = 0 an empty result
    z = tob.gemv(torch.empty(6, 0, dtype=torch.float16, device=cuda),
                 torch.empty(0, dtype=torch.float16, device=cuda))
    assert torch.equal(z, torch.zeros(6, dtype=torch.float16, device=cuda))
    assert tob.gemv(torch.empty(0, 8, device=cuda), torch.ones(8, device=cuda)).shape == (0,)


def test_gemv_errors(cuda):
    with pytest.raises(ValueError):
        tob.gemv(torch.zeros(2, 3, device=cuda), torch.zeros(2, 3, device=cuda))
    with pytest.raises(TypeError):
        tob.gemv(torch.zeros(2, 3, device=cuda), torch.zeros(3, device=cuda).half())
    with pytest.raises(ValueError):
        tob.gemv(torch.zeros(2, 3, dtype=torch.int32, device=cuda),
                 torch.zeros(3, dtype=torch.int32, device=cuda))
    with pytest.raises(ValueError):
        tob.gemv(torch.zeros(2, 3, device=cuda), torch.zeros(3, device=cuda),
                 out=torch.zeros(3, device=cuda))
    with pytest.raises(TypeError):
        tob.gemv(torch.zeros(2, 3, device=cuda), torch.zeros(3, device=cuda),
                 out=torch.zeros(2, dtype=torch.float16, device=cuda))
