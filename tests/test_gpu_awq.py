"""GPU parity of the AWQ kernels: pack/unpack/dequant bit-exact against the reference's
outputs, GEMV/GEMM within rtol=atol=1e-2 of the fp32-accumulated oracle (the tolerance the
path is specified to)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tileops_b200 as tob
from oracle import awq as oawq
from oracle import fused as ofused

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2
_DT = {"f16": torch.float16, "bf16": torch.bfloat16}


def make_awq(k, n, g, dtype, gen, lo=0.002, hi=0.02):
    """AWQ weights as the workloads specify them: int4 U{0..15}, zeros U{0..15},
    scales U(lo, hi), packed in AWQ order (oracle packer, checked against the reference)."""
    w = torch.randint(0, 16, (k, n), generator=gen, dtype=torch.int64)
    z = torch.randint(0, 16, (k // g, n), generator=gen, dtype=torch.int64)
    s = (torch.rand(k // g, n, generator=gen) * (hi - lo) + lo).to(dtype)
    qw = torch.from_numpy(oawq.pack(w.numpy()))
    qz = torch.from_numpy(oawq.pack(z.numpy()))
    return qw, s, qz


def test_pack_unpack_golden(cuda, golden):
    g = golden("awq.npz")
    c = g["roundtrip"]
    packed = tob.pack_awq_int4(c.tensor("x", cuda))
    assert packed.dtype == torch.int32
    assert np.array_equal(packed.cpu().numpy(), c["packed"])
    back = tob.unpack_awq_int4(packed)
    assert back.dtype == torch.int64
    assert np.array_equal(back.cpu().numpy(), c["unpacked"])
    c = g["pack_wide"]
    assert np.array_equal(tob.pack_awq_int4(c.tensor("x", cuda)).cpu().numpy(), c["packed"])


def test_pack_unpack_roundtrip_int32_and_int64(cuda):
    g = torch.Generator().manual_seed(3)
    x = torch.randint(0, 16, (33, 8 * 129), generator=g, dtype=torch.int64)
    for dt in (torch.int64, torch.int32):
        p = tob.pack_awq_int4(x.to(dt).to(cuda))
        assert np.array_equal(p.cpu().numpy(), oawq.pack(x.numpy()))
        assert torch.equal(tob.unpack_awq_int4(p).cpu(), x)
        assert torch.equal(tob.unpack_awq_int4(p.to(torch.int64)).cpu(), x)


@pytest.mark.parametrize("name", ["dequant_f16", "dequant_fullk", "dequant_bf16", "dequant_f32"])
def test_dequant_golden(cuda, golden, name):
    c = golden("awq.npz")[name]
    out = tob.awq_dequantize(c.tensor("qweight", cuda), c.tensor("scales", cuda),
                             c.tensor("qzeros", cuda))
    assert out.shape == tuple(c["out"].shape)
    assert np.array_equal(out.float().cpu().numpy(), c["out"])


@pytest.mark.parametrize("name", ["gemm_f16", "gemm_f16_m1", "gemm_f16_m3", "gemm_bf16",
                                  "gemm_bf16_m1", "gemm_f16_fullk"])
def test_gemm_golden(cuda, golden, name):
    c = golden("awq.npz")[name]
    y = tob.awq_gemm(c.tensor("x", cuda), c.tensor("qweight", cuda), c.tensor("scales", cuda),
                     c.tensor("qzeros", cuda), 1)
    assert y.dtype == c.tensor("scales").dtype
    np.testing.assert_allclose(y.float().cpu().numpy(), c["y"], rtol=RTOL, atol=ATOL)


def test_split_k_invariance(cuda, golden):
    c = golden("awq.npz")["gemm_splitk"]
    args = [c.tensor(f, cuda) for f in ("x", "qweight", "scales", "qzeros")]
    y1 = tob.awq_gemm(*args, split_k_iters=1)
    y4 = tob.awq_gemm(*args, split_k_iters=4)
    assert torch.equal(y1, y4)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,k,n,g", [
    (1, 4096, 4096, 128),     # decode GEMV (the [1,4096] x [4096,4096] G=128 layer)
    (1, 4096, 6144, 128),     # qkv
    (2, 14336, 4096, 128),    # down
    (4, 4096, 28672, 128),    # gate_up
    (3, 512, 136, 32),        # ragged column count (17 words)
    (1, 256, 64, 64),
    (16, 4096, 4096, 128),
    (64, 1024, 2048, 128),
    (5, 96, 64, 96),          # G == K not a multiple of 16
])
def test_gemm_vs_oracle(cuda, dtype, m, k, n, g):
    gen = torch.Generator().manual_seed(m * 131 + k + n)
    qw, s, qz = make_awq(k, n, g, _DT[dtype], gen)
    x = torch.randn(m, k, generator=gen).to(_DT[dtype])
    y = tob.awq_gemm(x.to(cuda), qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    want = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), dtype)
    np.testing.assert_allclose(y.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,k,n,g", [
    (128, 512, 768, 32),      # two quantisation groups per K block
    (300, 1024, 1024, 64),    # M tail
    (33, 4096, 256, 4096),    # one group over the whole K
    (512, 8192, 1024, 128),   # the 70B-class up-projection shape, narrowed in N
    (256, 200, 512, 200),     # K tail (K not a multiple of the K block), G == K
])
def test_gemm_tensor_core_vs_oracle(cuda, dtype, m, k, n, g):
    gen = torch.Generator().manual_seed(m + k * 3 + n)
    qw, s, qz = make_awq(k, n, g, _DT[dtype], gen)
    x = torch.randn(m, k, generator=gen).to(_DT[dtype])
    y = tob.awq_gemm(x.to(cuda), qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    want = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), dtype)
    np.testing.assert_allclose(y.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)


def test_gemm_prefill_full_size_sampled(cuda):
    """M=2048, K=8192, N=28672 bf16 (G=128): rows and columns sampled against the oracle."""
    m, k, n, g = 2048, 8192, 28672, 128
    gen = torch.Generator().manual_seed(1234 + 3)
    qw, s, qz = make_awq(k, n, g, torch.bfloat16, gen)
    x = torch.randn(m, k, generator=gen).bfloat16()
    y = tob.awq_gemm(x.to(cuda), qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    rows = torch.randperm(m, generator=gen)[:24].sort().values
    words = torch.randperm(n // 8, generator=gen)[:40].sort().values
    cols = (words[:, None] * 8 + torch.arange(8)[None, :]).reshape(-1)
    want = oawq.gemm(x[rows].float().numpy(), qw[:, words].numpy(), s[:, cols].float().numpy(),
                     qz[:, words].numpy(), "bf16")
    got = y[rows.to(cuda)][:, cols.to(cuda)].float().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_gemm_deterministic(cuda):
    gen = torch.Generator().manual_seed(9)
    qw, s, qz = make_awq(4096, 4096, 128, torch.float16, gen)
    x = torch.randn(1, 4096, generator=gen).half()
    args = (x.to(cuda), qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    y0 = tob.awq_gemm(*args)
    for _ in range(3):
        assert torch.equal(tob.awq_gemm(*args), y0)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,k,n,g", [
    # TMA-fed register-MMA kernel (3 <= M <= 64, N % 32 == 0, K % 64 == 0)
    (3, 4096, 28672, 128),    # 32-word column tiles, K split 4
    (4, 14336, 4096, 128),    # long K: the stage ring wraps, K split 8
    (8, 4096, 4096, 64),      # one full 8-token tile
    (9, 2048, 1024, 128),     # two token tiles, 7 of the second padded
    (16, 1024, 2048, 32),     # group size 32: several group rows per stage
    (24, 512, 512, 512),      # four token tiles, G == K
    (32, 1024, 4096, 128),    # the largest M it takes
    (32, 14336, 256, 128),    # 32 tokens of a long K chunk do not fit: two 16-token launches
    (20, 14336, 512, 128),    # the same with a 4-token second launch
    (64, 4096, 4096, 128),    # 33..64 tokens: eight token tiles (few tcgen05 tiles here)
    (48, 2048, 1024, 64),
    (40, 14336, 512, 128),    # x of a long K chunk does not fit: 32 + 8 tokens
    (33, 200, 256, 200),      # K % 64 != 0: the tcgen05 kernel takes it instead
    (5, 256, 96, 256),        # 12 words: a partial column tile, G == K
    # prefetching SIMT stream (M <= 2 below the decode kernel's layer size)
    (1, 4096, 4096, 128),     # the GEMV layer: 32 tiles x K split 8
    (2, 4096, 6144, 64),      # two tokens, 48 tiles
    (1, 1024, 2048, 32),      # 256-row chunks, eight groups per chunk
    (1, 3072, 1024, 3072),    # K split 6, one group over all chunks (G == K)
    (2, 3200, 2048, 128),     # K split 7, the last chunk 128 rows: idle warps
    (1, 4096, 28672, 128),    # 32-word column tiles
    (1, 2432, 1040, 128),     # 130 words (partial tile), K split 5: slices of ceil(128 / 5)
    (2, 14336, 4096, 128),    # several row blocks per warp
    (3, 1000, 256, 1000),     # K % 64 != 0, K tail inside the last row block
    (2, 100, 64, 100),        # K not a multiple of 8 (scalar x staging), G == K
    (1, 64, 16, 32),          # N = 16: 2 words per row
    (4, 2048, 4112, 64),      # N % 32 != 0: a partial 16-word column tile
    # general streaming kernel (M > 4 on shapes the TMA kernel does not take)
    (6, 200, 96, 200),
])
def test_gemv_small_m_vs_oracle(cuda, dtype, m, k, n, g):
    """The small-M kernels over their tile, token-tile, K-split, group and tail cases."""
    gen = torch.Generator().manual_seed(m * 7 + k + 3 * n)
    qw, s, qz = make_awq(k, n, g, _DT[dtype], gen)
    x = torch.randn(m, k, generator=gen).to(_DT[dtype])
    y = tob.awq_gemm(x.to(cuda), qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    want = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), dtype)
    np.testing.assert_allclose(y.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)


def test_gemv_launch_overlap_chain(cuda):
    """A chain of dependent small-M calls (each output is the next input) gives bit-identical
    results with launch overlap on and off, eagerly and replayed from a CUDA graph."""
    gen = torch.Generator().manual_seed(21)
    dims = [4096, 2048, 4096, 1024, 4096]
    layers = []
    for k, n in zip(dims[:-1], dims[1:]):
        qw, s, qz = make_awq(k, n, 128, torch.float16, gen, lo=0.0005, hi=0.002)
        layers.append((qw.to(cuda), s.to(cuda), qz.to(cuda)))
    x = torch.randn(2, dims[0], generator=gen).half().to(cuda)
    torch.cuda.synchronize()

    def chain(v):
        for qw, s, qz in layers:
            v = tob.awq_gemm(v, qw, s, qz, 1)
        return v

    prev = tob.set_launch_overlap(False)
    try:
        ref = chain(x)
        tob.set_launch_overlap(True)
        for _ in range(3):
            assert torch.equal(chain(x), ref)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            chain(x)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = chain(x)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        del graph
    finally:
        tob.set_launch_overlap(prev)
    want = x.float().cpu().numpy()
    for qw, s, qz in layers:
        want = oawq.gemm(want, qw.cpu().numpy(), s.float().cpu().numpy(), qz.cpu().numpy(), "f16")
    np.testing.assert_allclose(ref.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,k,n,g", [
    # stream-K decode kernel (1 <= M <= 32): column tiles of 256 split over K across CTAs
    (2, 4096, 28672, 128),    # two tokens on a wide layer (112 tiles x 16 K units)
    (3, 4096, 4096, 128),     # 16 tiles x 16 K units over 128 CTAs: 8 CTAs per tile
    (7, 4096, 6144, 64),      # scaled every 64 rows
    (16, 14336, 4096, 128),   # the down projection: 56 K units per tile
    (31, 4096, 28672, 32),    # four token tiles, scaled every 32 rows
    (12, 4096, 1056, 4096),   # G == K; a partial last column tile (1056 = 4 x 256 + 32)
    (2, 320, 256, 64),        # K % 256 != 0: the last K unit is partly outside the tensor
    (32, 1024, 512, 128),     # a tile split over several CTAs, each holding two units
])
def test_decode_kernel_vs_oracle(cuda, dtype, m, k, n, g):
    gen = torch.Generator().manual_seed(m * 11 + k + 5 * n + g)
    qw, s, qz = make_awq(k, n, g, _DT[dtype], gen)
    x = torch.randn(m, k, generator=gen).to(_DT[dtype])
    args = (x.to(cuda), qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    y = tob.awq_gemm(*args)
    want = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), dtype)
    np.testing.assert_allclose(y.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    assert torch.equal(tob.awq_gemm(*args), y)  # the partial sums are added in a fixed order


def test_decode_kernel_graph_replays_with_new_inputs(cuda):
    """One decode call captured in a CUDA graph and replayed with fresh activations: the
    per-launch flags of the cross-CTA partial sums are consumed and reset on every replay."""
    gen = torch.Generator().manual_seed(33)
    qw, s, qz = (t.to(cuda) for t in make_awq(4096, 4096, 128, torch.float16, gen))
    x = torch.zeros(16, 4096, dtype=torch.float16, device=cuda)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        tob.awq_gemm(x, qw, s, qz, 1)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = tob.awq_gemm(x, qw, s, qz, 1)
    for i in range(4):
        x.copy_(torch.randn(16, 4096, generator=gen).half())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, tob.awq_gemm(x, qw, s, qz, 1)), i
    del graph


@pytest.mark.parametrize("act", ["silu", "gelu"])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,k,n,g", [
    (1, 4096, 28672, 128),    # decode kernel, activation in its epilogue
    (16, 4096, 28672, 128),   # the decode step's gate_up
    (5, 1024, 1056, 64),      # a partial last column tile
    (32, 512, 512, 128),      # tiles split over several CTAs
    (2, 512, 528, 128),       # N % 32 != 0: GEMM into the workspace, then the activation
    (48, 8192, 2048, 128),    # stream-K tensor-core kernel, activation in its epilogue
    (48, 1024, 2048, 128),    # register-MMA GEMM + activation
    (300, 1024, 4096, 128),   # tensor-core GEMM + activation
])
def test_gemm_act_equals_gemm_then_act(cuda, act, dtype, m, k, n, g):
    """The gate_up linear with its activation equals the GEMM on the same (interleaved) weights
    followed by silu_and_mul / gelu_and_mul on its gate and up blocks, bit for bit; and the
    GEMM on the original weights + the activation, and the oracle, within the GEMM tolerance
    (the kernels' fp32 summation order depends on a column's tile, which the interleaving
    moves)."""
    gen = torch.Generator().manual_seed(m * 7 + k + 3 * n + g + (act == "gelu"))
    qw, s, qz = make_awq(k, n, g, _DT[dtype], gen)
    x = torch.randn(m, k, generator=gen).to(_DT[dtype])
    qw_i, s_i, qz_i = (t.to(cuda) for t in tob.awq_interleave_gate_up(qw, s, qz))
    xd = x.to(cuda)
    fused = tob.awq_gemm_silu_and_mul if act == "silu" else tob.awq_gemm_gelu_and_mul
    act_mul = tob.silu_and_mul if act == "silu" else tob.gelu_and_mul
    y = fused(xd, qw_i, s_i, qz_i)
    assert y.shape == (m, n // 2) and y.dtype == _DT[dtype]
    # the same GEMM, unfused: blocks of 8 columns alternate gate, up
    yi = tob.awq_gemm(xd, qw_i, s_i, qz_i, 1).view(m, n // 16, 2, 8)
    gate = yi[:, :, 0, :].reshape(m, n // 2)
    up = yi[:, :, 1, :].reshape(m, n // 2)
    assert torch.equal(y, act_mul(gate, up))
    # the activation against the oracle's, on that GEMM output: within two 16-bit ulps, or an
    # absolute 2^-14 where gelu's 1 + tanh cancels (large negative gates, results near zero)
    mine = ofused.act_and_mul(gate.float().cpu().numpy(), up.float().cpu().numpy(), act, dtype)
    ulp2 = 2.0 ** -9 if dtype == "f16" else 2.0 ** -6
    np.testing.assert_allclose(y.float().cpu().numpy(), mine, rtol=ulp2, atol=2.0 ** -14)
    # the original layout's GEMM + activation, and the oracle GEMM + activation
    full = tob.awq_gemm(xd, qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    sep = act_mul(full[:, :n // 2], full[:, n // 2:])
    np.testing.assert_allclose(y.float().cpu().numpy(), sep.float().cpu().numpy(), rtol=5e-2,
                               atol=5e-2)
    want = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), dtype)
    ref = ofused.act_and_mul(want[:, :n // 2], want[:, n // 2:], act, dtype)
    np.testing.assert_allclose(y.float().cpu().numpy(), ref, rtol=5e-2, atol=5e-2)
    assert torch.equal(fused(xd, qw_i, s_i, qz_i), y)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,k,n,g", [
    # stream-K tensor-core kernel (33 <= M <= 128, K >= 8192, at most 32 column tiles): 64-row
    # K blocks of 256-column tiles split over all SMs, later K ranges left as fp32 sums for the
    # tile's owner
    (33, 8192, 4096, 128),    # 16 tiles x 128 K blocks over 148 CTAs
    (64, 14336, 4096, 128),   # the decode step's down projection at 64 tokens
    (100, 8192, 1056, 64),    # a partial last column tile
    (128, 8192, 2048, 32),    # two scale rows per K block, a full 128-row x block
    (40, 8200, 256, 8200),    # K % 64 != 0 (zero-filled tail), G == K
    (77, 8192, 768, 32),
    (48, 8192, 256, 128),     # one tile over 32 CTAs: 31 partial sums added by its owner
    (65, 8192, 512, 64),
])
def test_stream_k_vs_oracle(cuda, dtype, m, k, n, g):
    gen = torch.Generator().manual_seed(m * 5 + k + 7 * n + g)
    qw, s, qz = make_awq(k, n, g, _DT[dtype], gen)
    x = torch.randn(m, k, generator=gen).to(_DT[dtype])
    args = (x.to(cuda), qw.to(cuda), s.to(cuda), qz.to(cuda), 1)
    y = tob.awq_gemm(*args)
    want = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), dtype)
    np.testing.assert_allclose(y.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    assert torch.equal(tob.awq_gemm(*args), y)  # the partial sums are added in a fixed order


def test_stream_k_graph_replays_with_new_inputs(cuda):
    """The stream-K kernel captured in a CUDA graph and replayed with fresh activations: the
    owners consume and reset the per-launch flags of the partial sums on every replay."""
    gen = torch.Generator().manual_seed(35)
    qw, s, qz = (t.to(cuda) for t in make_awq(8192, 2048, 128, torch.float16, gen))
    x = torch.zeros(64, 8192, dtype=torch.float16, device=cuda)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        tob.awq_gemm(x, qw, s, qz, 1)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = tob.awq_gemm(x, qw, s, qz, 1)
    for i in range(4):
        x.copy_(torch.randn(64, 8192, generator=gen).half())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, tob.awq_gemm(x, qw, s, qz, 1)), i
    del graph


@pytest.mark.parametrize("m,k,n", [(16, 4096, 4096), (4, 4096, 6144), (1, 4096, 4096),
                                   (48, 1024, 2048)])
def test_gemm_strided_input_read_in_place(cuda, m, k, n):
    """A row-strided slice of a wider activation (the o projection's input from a fused qkv
    output): the decode kernel reads it in place through its tensor map, other paths copy it
    first; the result equals the contiguous input's bit for bit."""
    gen = torch.Generator().manual_seed(m + k + n)
    qw, s, qz = (t.to(cuda) for t in make_awq(k, n, 128, torch.float16, gen))
    wide = torch.randn(m, k + 2048, generator=gen).half().to(cuda)
    x = wide[:, :k]
    assert m == 1 or not x.is_contiguous()  # one row of a slice is contiguous
    y = tob.awq_gemm(x, qw, s, qz, 1)
    assert torch.equal(y, tob.awq_gemm(x.contiguous(), qw, s, qz, 1))
