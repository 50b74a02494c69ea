"""N-sharded layers on CPU ranks of a world-size-2 gloo group: the sharding and all-gather
bookkeeping of tileops_b200.sharded, with the oracle standing in for the per-rank kernel, and
host-side failure detection (a rank that leaves before the collective)."""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _awq_compute(x, qw, s, qz):
    from oracle import awq as oawq

    y = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), "f16")
    return torch.from_numpy(y).to(torch.float16)


def _w8a8_compute(a, b, a_s, b_s, bs, od):
    from oracle import int8 as oi8

    y = oi8.block_matmul(a.numpy(), b.numpy(), a_s.numpy(), b_s.numpy(), tuple(bs), "f32")
    return torch.from_numpy(y).to(od)


def _worker(rank, world, port, case, q):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        timeout = timedelta(seconds=5 if case == "rank_exits" else 60)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
        from oracle import awq as oawq
        from oracle import int8 as oi8
        from tileops_b200 import sharded

        g = torch.Generator().manual_seed(7)  # every rank builds the same full layer
        if case == "awq":
            k, n, gs, m = 256, 512, 64, 5
            w = torch.randint(0, 16, (k, n), generator=g)
            z = torch.randint(0, 16, (k // gs, n), generator=g)
            s = (torch.rand(k // gs, n, generator=g) * 0.018 + 0.002).half()
            qw = torch.from_numpy(oawq.pack(w.numpy()))
            qz = torch.from_numpy(oawq.pack(z.numpy()))
            x = torch.randn(m, k, generator=g).half()
            layer = sharded.ShardedAWQLinear(qw, s, qz, compute=_awq_compute)
            assert layer.qweight.shape == (k, n // 8 // world)
            y = layer(x)
            yp = layer(x, layout="pmn")
            full = oawq.gemm(x.float().numpy(), qw.numpy(), s.float().numpy(), qz.numpy(), "f16")
            assert y.shape == (m, n)
            assert np.array_equal(y.float().numpy(), full)
            assert yp.shape == (world, m, n // world)
            assert np.array_equal(yp.permute(1, 0, 2).reshape(m, n).float().numpy(), full)
        elif case in ("w8a8_channel", "w8a8_tensor"):
            m, n, k = 6, 64, 128
            a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
            b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
            a_s = torch.rand(m, 1, generator=g) * 0.05 + 0.001
            if case == "w8a8_channel":
                bs, b_s = [1, k], torch.rand(n, 1, generator=g) * 0.01 + 0.001
            else:
                bs, b_s = [n, k], torch.rand(1, 1, generator=g) * 0.01 + 0.001
            layer = sharded.ShardedW8A8Linear(b, b_s, bs, output_dtype=torch.float32,
                                              compute=_w8a8_compute)
            y = layer(a, a_s)
            full = oi8.block_matmul(a.numpy(), b.numpy(), a_s.numpy(), b_s.numpy(), tuple(bs), "f32")
            np.testing.assert_allclose(y.numpy(), full, rtol=1e-6, atol=1e-6)
        elif case == "rank_exits":
            # Rank 1 leaves between steps, before the gather; rank 0 must get an error from
            # its next collective (process-group timeout), not hang.
            local = torch.full((2, 4), float(rank))
            if rank == 1:
                q.put((rank, "left"))
                return
            try:
                sharded.gather_columns(local)
            except Exception as e:  # noqa: BLE001 - any backend error is the expected outcome
                q.put((rank, "error:" + type(e).__name__))
                return
            q.put((rank, "no error"))
            return
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


def _run(case, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=timeout) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("case", ["awq", "w8a8_channel", "w8a8_tensor"])
def test_sharded_matches_unsharded(case):
    res = _run(case)
    assert res == {0: "ok", 1: "ok"}, res


def test_rank_that_leaves_is_detected():
    res = _run("rank_exits")
    assert res[1] == "left"
    assert res[0].startswith("error:"), res


def test_shard_bounds_validation():
    from tileops_b200.sharded import shard_bounds, shard_w8a8

    assert shard_bounds(28672, 3, 8, 8) == (10752, 14336)
    with pytest.raises(ValueError):
        shard_bounds(100, 0, 8, 8)
    w = torch.zeros(64, 16, dtype=torch.int8)
    with pytest.raises(ValueError):
        shard_w8a8(w, torch.ones(3, 1), 24, 1, 2)  # 32-row shards do not align with 24-row blocks


def test_from_shard_single_rank_gathered_is_local():
    """Without a process group a layer is its own shard and `gathered` is the local call."""
    from tileops_b200.sharded import ShardedAWQLinear

    calls = []

    def compute(x, qw, s, qz):
        calls.append((x.shape, qw.shape, s.shape, qz.shape))
        return torch.full((x.shape[0], s.shape[1]), 2.0)

    qw = torch.zeros(64, 4, dtype=torch.int32)
    s = torch.ones(1, 32, dtype=torch.float16)
    qz = torch.zeros(1, 4, dtype=torch.int32)
    layer = ShardedAWQLinear.from_shard(qw, s, qz, compute=compute)
    assert (layer.rank, layer.world, layer.n) == (0, 1, 32)
    y = layer.gathered(torch.zeros(3, 64))
    assert y.shape == (3, 32) and bool((y == 2.0).all())
    assert calls == [((3, 64), (64, 4), (1, 32), (1, 4))]
    layer.close()  # nothing was mapped


def test_ipc_handle_length_checked_before_the_library():
    import tileops_b200._lib as lib

    with pytest.raises(ValueError):
        lib.ipc_open(b"\x00" * 10)
