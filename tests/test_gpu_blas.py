"""GPU parity of the dense 16-bit GEMM (tileops.gemm / mm): the tcgen05 tiles with B read
MN-major against an fp32 torch product of the same inputs (rtol = atol = 1e-2 on outputs of unit
scale), ragged shapes, out= and the library fallback for other shapes."""

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


def test_gemm_other_shapes_and_errors(cuda):
    a, b = _inputs(33, 50, 20, torch.float16, 4)  # N % 64 != 0: library GEMM
    c = tob.gemm(a.to(cuda), b.to(cuda))
    np.testing.assert_allclose(c.float().cpu().numpy(), (a.float() @ b.float()).numpy(),
                               rtol=1e-2, atol=1e-2)
    with pytest.raises(ValueError):
        tob.gemm(torch.zeros(2, 3, device=cuda), torch.zeros(4, 5, device=cuda))
    with pytest.raises(TypeError):
        tob.gemm(torch.zeros(2, 3, device=cuda), torch.zeros(3, 5, device=cuda).half())
    with pytest.raises(ValueError):
        tob.gemm(torch.zeros(3, device=cuda), torch.zeros(3, 5, device=cuda))
