"""The allocation-free tensor-wide FP8 quantiser, called through the C ABI.

`to_input_to_fp8_noalloc` exists for callers that cannot give the library device memory: a
serving runtime that has reserved all device memory for its own pool (a cudaMalloc while it
serves would fail or fragment that pool), or a foreign-language binding that only passes tensor
pointers and owns no device allocator. Its scratch is built into the library, so it must match
the workspace-taking entry point `to_input_to_fp8` bit for bit, including on back-to-back calls
that reuse that built-in scratch with different inputs, and it must refuse inputs larger than
its scratch covers.

This file is collected after every other test file on purpose.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import tileops_b200 as tob
from tileops_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_ELEMS = 8192 * 16384  # the scratch limit stated in include/tileops_b200.h


def _noalloc(x: torch.Tensor):
    """Calls the entry point directly through ctypes, as a C caller would."""
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty((), dtype=torch.float32, device=x.device)
    rc = _lib.load().to_input_to_fp8_noalloc(
        ctypes.c_void_p(x.data_ptr()), _lib.DTYPE_CODES[x.dtype], x.numel(),
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(s.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.TO_OK, _lib.last_error()
    return q, s


def _same(a_q, a_s, b_q, b_s):
    # The tolerance of the quantiser tests: codes and the dequant scale are bit-exact (a NaN
    # scale, from a NaN input, matches a NaN scale).
    assert np.array_equal(a_q.view(torch.uint8).cpu().numpy(), b_q.view(torch.uint8).cpu().numpy())
    assert np.array_equal(a_s.cpu().numpy(), b_s.cpu().numpy(), equal_nan=True)


def test_noalloc_matches_workspace_entry_two_calls_in_a_row(cuda):
    g = torch.Generator().manual_seed(77)
    # First call: a large bf16 tensor (many partial maxima); second call: a smaller fp32 tensor
    # with a much smaller range, so stale partial maxima from the first call would show up.
    x1 = (torch.randn(4096, 3001, generator=g) * 5.0).to(torch.bfloat16).to(cuda)
    x2 = (torch.randn(70001, generator=g) * 0.01).to(cuda)
    q1, s1 = _noalloc(x1)
    q2, s2 = _noalloc(x2)
    r1, rs1 = tob.input_to_float8(x1)
    r2, rs2 = tob.input_to_float8(x2)
    torch.cuda.synchronize()
    _same(q1, s1, r1, rs1)
    _same(q2, s2, r2, rs2)
    # and once more in the other order, with an fp16 input that is not 16-byte aligned
    x3 = (torch.randn(1 + 123457, generator=g) * 3.0).half().to(cuda)[1:]
    q3, s3 = _noalloc(x3)
    q1b, s1b = _noalloc(x1)
    r3, rs3 = tob.input_to_float8(x3)
    _same(q3, s3, r3, rs3)
    _same(q1b, s1b, r1, rs1)


def test_noalloc_nan_input_then_a_clean_one(cuda):
    # A NaN makes the scale NaN; the next call must not see that NaN left in the scratch.
    g = torch.Generator().manual_seed(78)
    x1 = torch.randn(50000, generator=g).to(torch.bfloat16)
    x1[12345] = float("nan")
    x1 = x1.to(cuda)
    x2 = (torch.randn(3000, generator=g) * 0.5).to(cuda)
    q1, s1 = _noalloc(x1)
    q2, s2 = _noalloc(x2)
    r1, rs1 = tob.input_to_float8(x1)
    r2, rs2 = tob.input_to_float8(x2)
    assert torch.isnan(s1).item()
    _same(q1, s1, r1, rs1)
    _same(q2, s2, r2, rs2)


def test_noalloc_rejects_inputs_beyond_its_scratch(cuda):
    x = torch.zeros(16, device=cuda)
    q = torch.empty(16, dtype=torch.float8_e4m3fn, device=cuda)
    s = torch.empty((), device=cuda)
    # The size is checked before any memory is touched, so a small buffer is enough here.
    rc = _lib.load().to_input_to_fp8_noalloc(
        ctypes.c_void_p(x.data_ptr()), _lib.DTYPE_CODES[x.dtype], MAX_ELEMS + 1,
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(s.data_ptr()), None)
    assert rc == _lib.TO_EINVAL
    assert "scratch limit" in _lib.last_error()
    rc = _lib.load().to_input_to_fp8_noalloc(
        ctypes.c_void_p(x.data_ptr()), _lib.DTYPE_CODES[x.dtype], 0,
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(s.data_ptr()), None)
    assert rc == _lib.TO_EINVAL
