"""Failure detection on the GPU without a fault: the bounded waits of the tcgen05 pipelines give
up after their limit, record the timeout in the device error word and return, and the context
stays usable. The wait is made to run out on a barrier that nothing arrives at."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tileops_b200 as tob
import tileops_b200._lib as lib
from oracle import int8 as oi8

pytestmark = pytest.mark.gpu


def _selftest(cuda, limit_us: int, arrive: bool) -> tuple[int, int]:
    out = torch.zeros(2, dtype=torch.int64, device=cuda)
    lib.wait_limit_selftest(limit_us, arrive, out.data_ptr(),
                            torch.cuda.current_stream(cuda).cuda_stream)
    torch.cuda.synchronize(cuda)
    completed, waited_ns = (int(v) for v in out.cpu())
    return completed, waited_ns


def test_wait_completes_when_barrier_arrives(cuda):
    completed, waited_ns = _selftest(cuda, 1000, arrive=True)
    assert completed == 1
    assert waited_ns < 1_000_000
    assert lib.device_error_word(clear=True) == 0


def test_wait_gives_up_and_records_timeout(cuda):
    limit_us = 2000
    completed, waited_ns = _selftest(cuda, limit_us, arrive=False)
    assert completed == 0
    assert waited_ns >= limit_us * 1000
    assert waited_ns < 1_000_000_000
    assert lib.device_error_word(clear=True) == 1
    assert lib.device_error_word(clear=True) == 0


def test_context_usable_after_timeout(cuda):
    _selftest(cuda, 500, arrive=False)
    assert lib.device_error_word(clear=True) == 1
    g = torch.Generator().manual_seed(7)
    m, n, k = 200, 320, 1024
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8, generator=g)
    b = torch.randint(-127, 128, (n, k), dtype=torch.int8, generator=g)
    acc = tob.w8a8_int8_accumulators(a.to(cuda), b.to(cuda))
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), oi8.accumulators(a.numpy(),
                                                                               b.numpy()))


@pytest.mark.parametrize("limit_us", [0, -5, 1_000_001])
def test_limit_outside_range_rejected(cuda, limit_us):
    out = torch.zeros(2, dtype=torch.int64, device=cuda)
    with pytest.raises(ValueError):
        lib.wait_limit_selftest(limit_us, False, out.data_ptr(), 0)


def _barrier(flags: list[torch.Tensor], rank: int, counter: torch.Tensor, cuda) -> None:
    import ctypes

    table = (ctypes.c_void_p * len(flags))(*[f.data_ptr() for f in flags])
    lib.check(lib.load().to_peer_barrier(table, len(flags), rank, counter.data_ptr(),
                                         torch.cuda.current_stream(cuda).cuda_stream),
              "peer_barrier")
    torch.cuda.synchronize(cuda)


def test_peer_barrier_passes_when_every_rank_arrived(cuda):
    """Rank 0 of two, with rank 1's arrival already in rank 0's flags (one process, local
    memory standing in for the mapped arrays): the barrier completes, the count advances and
    rank 0's slot is raised in both arrays."""
    slots = lib.load().to_peer_flags_bytes() // 8
    flags = [torch.zeros(slots, dtype=torch.int64, device=cuda) for _ in range(2)]
    counter = torch.zeros(1, dtype=torch.int64, device=cuda)
    flags[0][1] = 1
    _barrier(flags, 0, counter, cuda)
    assert int(counter.item()) == 1
    assert int(flags[0][0].item()) == 1 and int(flags[1][0].item()) == 1
    assert lib.device_error_word(clear=True) == 0


def test_peer_barrier_gives_up_on_a_rank_that_never_arrives(cuda):
    """Rank 1 never raises its slot: rank 0's bounded wait ends after the library's limit with
    the timeout code in the error word, and the context still runs a GEMM bit-exactly."""
    import time

    slots = lib.load().to_peer_flags_bytes() // 8
    flags = [torch.zeros(slots, dtype=torch.int64, device=cuda) for _ in range(2)]
    counter = torch.zeros(1, dtype=torch.int64, device=cuda)
    t0 = time.perf_counter()
    _barrier(flags, 0, counter, cuda)
    assert time.perf_counter() - t0 < 30.0
    assert lib.device_error_word(clear=True) == 1
    g = torch.Generator().manual_seed(8)
    a = torch.randint(-127, 128, (130, 512), dtype=torch.int8, generator=g)
    b = torch.randint(-127, 128, (256, 512), dtype=torch.int8, generator=g)
    acc = tob.w8a8_int8_accumulators(a.to(cuda), b.to(cuda))
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), oi8.accumulators(a.numpy(),
                                                                               b.numpy()))
