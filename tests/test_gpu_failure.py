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
