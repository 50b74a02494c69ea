"""GPU parity of the W8A8 INT8 and FP8 GEMMs: int32 accumulators bit-exact against the
exact integer GEMM, outputs within tolerance of the fp32-accumulated oracle, against the
reference's golden outputs, on the reference tests' ragged block shapes and on the
per-token x per-channel / per-tensor layouts of the large layers."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tileops_b200 as tob
from oracle import fp8 as ofp8
from oracle import int8 as oi8

pytestmark = pytest.mark.gpu

_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _f(t):
    return t.float().cpu().numpy()


def test_int8_golden_small(cuda, golden):
    c = golden("int8.npz")["w8a8_small"]
    y = tob.w8a8_block_int8_matmul(c.tensor("a", cuda), c.tensor("b", cuda), c.tensor("a_s", cuda),
                                   c.tensor("b_s", cuda), list(c["block"]),
                                   output_dtype=torch.float32)
    np.testing.assert_allclose(_f(y), c["c"], rtol=1e-4, atol=1e-4)


def test_int8_golden_channel(cuda, golden):
    c = golden("int8.npz")["w8a8_channel"]
    a, b = c.tensor("a", cuda), c.tensor("b", cuda)
    y = tob.w8a8_block_int8_matmul(a, b, c.tensor("a_s", cuda), c.tensor("b_s", cuda),
                                   list(c["block"]), output_dtype=torch.bfloat16)
    assert y.dtype == torch.bfloat16
    np.testing.assert_allclose(_f(y), c["c"], rtol=1e-2, atol=1e-2)
    acc = tob.w8a8_int8_accumulators(a, b)
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), c["acc"])


def test_int8_apply_linear_golden(cuda, golden):
    c = golden("int8.npz")["apply_linear"]
    y = tob.apply_w8a8_block_int8_linear(c.tensor("x", cuda), c.tensor("w", cuda),
                                         list(c["block"]), c.tensor("w_s", cuda),
                                         bias=c.tensor("bias", cuda))
    assert y.dtype == torch.float16
    np.testing.assert_allclose(_f(y), c["y"], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("m,n,k", [(256, 11008, 4096), (1, 64, 4096), (200, 1000, 512),
                                   (128, 256, 128), (300, 384, 1024), (17, 4097, 96)])
def test_int8_accumulators_bit_exact(cuda, m, n, k):
    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    acc = tob.w8a8_int8_accumulators(a.to(cuda), b.to(cuda))
    want = oi8.accumulators(a.numpy(), b.numpy())
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), want)


@pytest.mark.parametrize("out", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("m,n,k", [(256, 11008, 4096), (64, 512, 4096), (300, 384, 1024),
                                   (7, 100, 256)])
def test_int8_per_channel_vs_oracle(cuda, out, m, n, k):
    g = torch.Generator().manual_seed(m * n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand(m, 1, generator=g) * 0.045 + 0.005
    b_s = torch.rand(n, 1, generator=g) * 0.009 + 0.001
    y = tob.w8a8_block_int8_matmul(a.to(cuda), b.to(cuda), a_s.to(cuda), b_s.to(cuda), [1, k],
                                   output_dtype=_DT[out])
    want = oi8.block_matmul(a.numpy(), b.numpy(), a_s.numpy(), b_s.numpy(), (1, k), out)
    tol = 1e-4 if out == "f32" else 1e-2
    np.testing.assert_allclose(_f(y), want, rtol=tol, atol=tol)


@pytest.mark.parametrize("m,n,k,bn,bk", [(6, 10, 24, 4, 8), (33, 260, 512, 128, 128),
                                         (128, 256, 384, 128, 128)])
def test_int8_block_scaled_vs_oracle(cuda, m, n, k, bn, bk):
    g = torch.Generator().manual_seed(m + 3 * n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    kt = -(-k // bk)
    a_s = torch.rand(m, kt, generator=g) * 0.05 + 0.001
    b_s = torch.rand(-(-n // bn), kt, generator=g) * 0.05 + 0.001
    y = tob.w8a8_block_int8_matmul(a.to(cuda), b.to(cuda), a_s.to(cuda), b_s.to(cuda), [bn, bk],
                                   output_dtype=torch.float32)
    want = oi8.block_matmul(a.numpy(), b.numpy(), a_s.numpy(), b_s.numpy(), (bn, bk), "f32")
    np.testing.assert_allclose(_f(y), want, rtol=1e-4, atol=1e-4)


def test_fp8_golden_small(cuda, golden):
    c = golden("fp8.npz")["w8a8_small"]
    args = [c.tensor(f, cuda) for f in ("a", "b", "a_s", "b_s")]
    y = tob.w8a8_block_fp8_matmul(*args, list(c["block"]), output_dtype=torch.float32)
    y2 = tob.w8a8_triton_block_scaled_mm(*args, list(c["block"]), output_dtype=torch.float32)
    assert torch.equal(y, y2)
    np.testing.assert_allclose(_f(y), c["c"], rtol=1e-4, atol=1e-4)


def test_fp8_apply_linear_golden(cuda, golden):
    c = golden("fp8.npz")["apply_linear"]
    y = tob.apply_w8a8_block_fp8_linear(c.tensor("x", cuda), c.tensor("w", cuda),
                                        list(c["block"]), c.tensor("w_s", cuda),
                                        bias=c.tensor("bias", cuda))
    np.testing.assert_allclose(_f(y), c["y"], rtol=1e-3, atol=1e-3)


def test_fp8_layer_golden(cuda, golden):
    """Dynamic per-token quant of A, per-tensor quant of B, per-token x per-tensor GEMM."""
    c = golden("fp8.npz")["fp8_layer"]
    A, B = c.tensor("A", cuda), c.tensor("B", cuda)
    qa, sa = tob.per_token_group_quant_fp8(A, A.shape[1])
    qb, sb = tob.input_to_float8(B)
    assert np.array_equal(qa.view(torch.uint8).cpu().numpy(), c["qa"])
    assert np.array_equal(qb.view(torch.uint8).cpu().numpy(), c["qb"])
    y = tob.w8a8_block_fp8_matmul(qa, qb, sa, sb.reshape(1, 1), [B.shape[0], A.shape[1]],
                                  output_dtype=torch.bfloat16)
    np.testing.assert_allclose(_f(y), c["c"], rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("m,n,k", [(8192, 8192, 8192), (256, 512, 1024), (130, 200, 4096),
                                   (1, 128, 256)])
def test_fp8_per_token_per_tensor_vs_oracle(cuda, m, n, k):
    g = torch.Generator().manual_seed(m + n + k + 1)
    A = torch.randn(m, k, generator=g).to(torch.bfloat16)
    B = torch.randn(n, k, generator=g).to(torch.bfloat16)
    qa, sa = tob.per_token_group_quant_fp8(A.to(cuda), k)
    qb, sb = tob.input_to_float8(B.to(cuda))
    y = tob.w8a8_block_fp8_matmul(qa, qb, sa, sb.reshape(1, 1), [n, k], output_dtype=torch.bfloat16)
    if m * n * k > 2 ** 33:
        # Full-size check: a seeded sample of rows against the oracle.
        rows = torch.randperm(m, generator=g)[:64].sort().values
        want = ofp8.block_matmul(qa[rows].view(torch.uint8).cpu().numpy(),
                                 qb.view(torch.uint8).cpu().numpy(), sa[rows].cpu().numpy(),
                                 sb.reshape(1, 1).cpu().numpy(), (n, k), "bf16")
        got = _f(y[rows.to(cuda)])
    else:
        want = ofp8.block_matmul(qa.view(torch.uint8).cpu().numpy(), qb.view(torch.uint8).cpu().numpy(),
                                 sa.cpu().numpy(), sb.reshape(1, 1).cpu().numpy(), (n, k), "bf16")
        got = _f(y)
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("m,n,k", [(129, 320, 384), (256, 1000, 640), (200, 11008, 4096)])
def test_int8_ksplit_pair_vs_oracle(cuda, m, n, k):
    """128 < M <= 256 layers whose 256 x 160 tiles fit one wave of CTA pairs split K over a
    cluster pair (odd K-block counts included): int32 accumulators bit-exact, scaled outputs
    against the oracle, and identical results across calls."""
    g = torch.Generator().manual_seed(7 * m + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand(m, 1, generator=g) * 0.045 + 0.005
    b_s = torch.rand(n, 1, generator=g) * 0.009 + 0.001
    acc = tob.w8a8_int8_accumulators(a.to(cuda), b.to(cuda))
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), oi8.accumulators(a.numpy(), b.numpy()))
    args = (a.to(cuda), b.to(cuda), a_s.to(cuda), b_s.to(cuda), [1, k])
    y = tob.w8a8_block_int8_matmul(*args, output_dtype=torch.bfloat16)
    want = oi8.block_matmul(a.numpy(), b.numpy(), a_s.numpy(), b_s.numpy(), (1, k), "bf16")
    np.testing.assert_allclose(_f(y), want, rtol=1e-2, atol=1e-2)
    assert torch.equal(tob.w8a8_block_int8_matmul(*args, output_dtype=torch.bfloat16), y)


def test_int8_ksplit_pair_fused_bias(cuda):
    """apply_w8a8_block_int8_linear with an fp16 bias on a K-split pair: the bias is added
    after rounding to fp16 and rounded again, as in the reference."""
    from oracle.numerics import rounder

    m, n, k = 200, 1000, 512
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).half()
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    w_s = torch.rand(n, 1, generator=g) * 0.009 + 0.001
    bias = torch.randn(n, generator=g).half()
    y = tob.apply_w8a8_block_int8_linear(x.to(cuda), w.to(cuda), [1, k], w_s.to(cuda),
                                         bias=bias.to(cuda))
    q, s = oi8.group_quant(x.float().numpy(), k)
    mm = oi8.block_matmul(q, w.numpy(), s, w_s.numpy(), (1, k), "f16")
    want = rounder("f16")(mm + bias.float().numpy())
    np.testing.assert_allclose(_f(y), want, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("m,n,k", [(200, 3000, 1024), (256, 11008, 512)])
def test_fp8_ksplit_pair_vs_oracle(cuda, m, n, k):
    g = torch.Generator().manual_seed(m + n + 2 * k)
    A = torch.randn(m, k, generator=g).to(torch.bfloat16)
    B = torch.randn(n, k, generator=g).to(torch.bfloat16)
    qa, sa = tob.per_token_group_quant_fp8(A.to(cuda), k)
    qb, sb = tob.input_to_float8(B.to(cuda))
    y = tob.w8a8_block_fp8_matmul(qa, qb, sa, sb.reshape(1, 1), [n, k], output_dtype=torch.bfloat16)
    want = ofp8.block_matmul(qa.view(torch.uint8).cpu().numpy(), qb.view(torch.uint8).cpu().numpy(),
                             sa.cpu().numpy(), sb.reshape(1, 1).cpu().numpy(), (n, k), "bf16")
    np.testing.assert_allclose(_f(y), want, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("m,n,k", [(256, 11008, 4096), (200, 1000, 640)])
def test_int8_pair_accumulators_with_bf16_output(cuda, m, n, k):
    """The 2-CTA (cta_group::2) tiles take 128 < M <= 256 layers with a 16-bit output: the raw
    int32 accumulators they emit next to the bf16 output are bit-exact."""
    from tileops_b200.quant_int8 import _run_w8a8

    g = torch.Generator().manual_seed(3 * m + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a_s = torch.rand(m, 1, generator=g) * 0.045 + 0.005
    b_s = torch.rand(n, 1, generator=g) * 0.009 + 0.001
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda)
    y = _run_w8a8("to_w8a8_i8_gemm", "w8a8_block_int8_matmul", a.to(cuda), b.to(cuda), a_s.to(cuda),
                  b_s.to(cuda), 1, k, m, n, k, torch.bfloat16, acc_out=acc)
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), oi8.accumulators(a.numpy(), b.numpy()))
    want = oi8.block_matmul(a.numpy(), b.numpy(), a_s.numpy(), b_s.numpy(), (1, k), "bf16")
    np.testing.assert_allclose(_f(y), want, rtol=1e-2, atol=1e-2)


def test_int8_pair_launch_overlap_chain(cuda):
    """A chain of 2-CTA INT8 layers (each bf16 output quantised per token into the next
    layer's input) gives bit-identical results with launch overlap on and off, eagerly and
    replayed from a CUDA graph; the first layer also matches the oracle."""
    g = torch.Generator().manual_seed(33)
    m, dims = 200, [4096, 2048, 4096, 1024]
    layers = []
    for k, n in zip(dims[:-1], dims[1:]):
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
        w_s = torch.rand(n, 1, generator=g) * 0.002 + 0.0005
        layers.append((w.to(cuda), w_s.to(cuda)))
    x = (torch.randn(m, dims[0], generator=g) * 2).to(torch.bfloat16).to(cuda)
    torch.cuda.synchronize()

    def chain(v):
        outs = []
        for w, w_s in layers:
            q, q_s = tob.per_token_quant_int8(v)
            v = tob.w8a8_block_int8_matmul(q, w, q_s, w_s, [1, w.shape[1]],
                                           output_dtype=torch.bfloat16)
            outs.append(v)
        return outs

    prev = tob.set_launch_overlap(False)
    try:
        ref = chain(x)
        tob.set_launch_overlap(True)
        for _ in range(3):
            assert all(torch.equal(a, b) for a, b in zip(chain(x), ref))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            chain(x)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = chain(x)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert all(torch.equal(a, b) for a, b in zip(outs, ref))
        del graph
    finally:
        tob.set_launch_overlap(prev)
    q, q_s = tob.per_token_quant_int8(x)
    w, w_s = layers[0]
    want = oi8.block_matmul(q.cpu().numpy(), w.cpu().numpy(), q_s.cpu().numpy(),
                            w_s.cpu().numpy(), (1, dims[0]), "bf16")
    np.testing.assert_allclose(_f(ref[0]), want, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("m,n,k,bn", [(300, 384, 1024, 128),   # ragged M, 8 K blocks
                                      (256, 512, 448, 128),    # last K block half full
                                      (128, 640, 768, 256),    # column blocks span two tiles
                                      (200, 264, 512, 264)])   # one column block (bn = N)
def test_int8_block_scaled_tensor_core_vs_oracle(cuda, out, m, n, k, bn):
    """block_k = 128 with per-(row, K block) and per-(column block, K block) scales on the
    tcgen05 block-scaled tiles (two TMEM buffers folded into fp32 sums per K block)."""
    g = torch.Generator().manual_seed(m * 7 + n + k + bn)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    kt = -(-k // 128)
    a_s = torch.rand(m, kt, generator=g) * 0.05 + 0.001
    b_s = torch.rand(-(-n // bn), kt, generator=g) * 0.05 + 0.001
    y = tob.w8a8_block_int8_matmul(a.to(cuda), b.to(cuda), a_s.to(cuda), b_s.to(cuda), [bn, 128],
                                   output_dtype=_DT[out])
    want = oi8.block_matmul(a.numpy(), b.numpy(), a_s.numpy(), b_s.numpy(), (bn, 128), out)
    tol = 1e-4 if out == "f32" else 1e-2
    np.testing.assert_allclose(_f(y), want, rtol=tol, atol=tol)


@pytest.mark.parametrize("m,n,k,bn", [(256, 384, 1024, 128), (130, 256, 640, 256)])
def test_fp8_block_scaled_tensor_core_vs_oracle(cuda, m, n, k, bn):
    """The e4m3 block-scaled path (DeepSeek-style 128 x 128 blocks) on the tcgen05 tiles."""
    g = torch.Generator().manual_seed(m + 5 * n + k)
    qa = (torch.randn(m, k, generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    qb = (torch.randn(n, k, generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    kt = -(-k // 128)
    a_s = torch.rand(m, kt, generator=g) * 0.01 + 0.0005
    b_s = torch.rand(-(-n // bn), kt, generator=g) * 0.01 + 0.0005
    y = tob.w8a8_block_fp8_matmul(qa.to(cuda), qb.to(cuda), a_s.to(cuda), b_s.to(cuda), [bn, 128],
                                  output_dtype=torch.bfloat16)
    want = ofp8.block_matmul(qa.view(torch.uint8).numpy(), qb.view(torch.uint8).numpy(),
                             a_s.numpy(), b_s.numpy(), (bn, 128), "bf16")
    np.testing.assert_allclose(_f(y), want, rtol=1e-2, atol=1e-2)


def test_fp8_apply_linear_block_128_with_bias(cuda):
    """apply_w8a8_block_fp8_linear with [128, 128] blocks and a bf16 bias: group quantisation of
    the input, the block-scaled tensor-core GEMM, the bias added after rounding (fused)."""
    g = torch.Generator().manual_seed(77)
    m, n, k = 256, 512, 1024
    x = torch.randn(m, k, generator=g).bfloat16()
    w = (torch.randn(n, k, generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    w_s = torch.rand(n // 128, k // 128, generator=g) * 0.01 + 0.0005
    bias = torch.randn(n, generator=g).bfloat16()
    y = tob.apply_w8a8_block_fp8_linear(x.to(cuda), w.to(cuda), [128, 128], w_s.to(cuda),
                                        bias=bias.to(cuda))
    assert y.dtype == torch.bfloat16 and y.shape == (m, n)
    q, s = tob.per_token_group_quant_fp8(x.to(cuda), 128)
    mm = ofp8.block_matmul(q.view(torch.uint8).cpu().numpy(), w.view(torch.uint8).numpy(),
                           s.cpu().numpy(), w_s.numpy(), (128, 128), "bf16")
    want = (torch.from_numpy(mm).bfloat16() + bias).float().numpy()
    np.testing.assert_allclose(_f(y), want, rtol=1e-2, atol=1e-2)
