"""The C-ABI library loads, exports exactly what include/tileops_b200.h declares, and the
facade validates arguments like the reference before touching a device. No GPU needed:
no entry point that launches a kernel is called here."""

from __future__ import annotations

import ctypes
import re
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import tileops_b200 as tob
from tileops_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "tileops_b200.h"


def _declared() -> dict[str, int]:
    text = HEADER.read_text()
    out = {}
    for m in re.finditer(r"TO_API\s+[\w\s\*]+?\b(to_\w+)\s*\(([^)]*)\)", text):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else len(args.split(","))
    return out


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from tileops_b200 import build

        build.build()
    return _lib.load()


def test_header_declares_entry_points():
    decl = _declared()
    assert len(decl) >= 20
    for name in ("to_awq_gemm", "to_w8a8_i8_gemm", "to_w8a8_fp8_gemm", "to_input_to_fp8",
                 "to_per_token_group_quant_fp8", "to_quant_per_channel_i8"):
        assert name in decl


def test_every_declared_symbol_is_exported(lib):
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_signature_table_matches_header():
    decl = _declared()
    assert set(decl) == set(_lib.SIGNATURES), set(decl) ^ set(_lib.SIGNATURES)
    for name, nargs in decl.items():
        assert len(_lib.SIGNATURES[name][1]) == nargs, name


def test_version_and_error_string(lib):
    assert "sm_100a" in _lib.version()
    assert isinstance(_lib.last_error(), str)


def test_workspace_queries_need_no_device(lib):
    assert lib.to_input_quant_workspace_size() >= 4
    assert lib.to_awq_gemm_workspace_size(1, 4096, 4096, 128) >= 0


def test_gemv_shape_checks_need_no_device(lib):
    assert lib.to_gemv(None, None, None, _lib.DTYPE_CODES[torch.float16], -1, 4, None) == \
        _lib.TO_EINVAL
    assert lib.to_gemv(None, None, None, _lib.DTYPE_CODES[torch.float16], 0, 4, None) == _lib.TO_OK
    assert lib.to_gemv(None, None, None, _lib.DTYPE_CODES[torch.float16], 3, 4, None) == \
        _lib.TO_EINVAL  # null pointers


def test_status_mapping():
    with pytest.raises(ValueError):
        _lib.check(_lib.TO_EINVAL, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.TO_EUNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.TO_ECUDA, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.TO_ETIMEOUT, "x")


def test_cpu_tensors_are_rejected_not_computed():
    x = torch.randn(4, 16)
    with pytest.raises(TypeError, match="CUDA"):
        tob.per_token_quant_int8(x)
    with pytest.raises(TypeError, match="CUDA"):
        tob.input_to_float8(x)
    with pytest.raises(TypeError, match="CUDA"):
        tob.pack_awq_int4(torch.zeros(2, 8, dtype=torch.int64))


def test_reference_validation_order():
    # Shape / value errors the reference raises before any compute.
    with pytest.raises(ValueError, match="divisible by 8"):
        tob.pack_awq_int4(torch.zeros(2, 7, dtype=torch.int64))
    with pytest.raises(TypeError, match="int32"):
        tob.unpack_awq_int4(torch.zeros(2, 7, dtype=torch.float32))
    with pytest.raises(ValueError, match="must be 2-D"):
        tob.awq_gemm(torch.zeros(4), torch.zeros(4, 1, dtype=torch.int32),
                     torch.zeros(1, 8), torch.zeros(1, 1, dtype=torch.int32), 1)
    with pytest.raises(ValueError, match="power of 2"):
        tob.awq_gemm(torch.zeros(1, 32), torch.zeros(32, 8, dtype=torch.int32),
                     torch.zeros(1, 64, dtype=torch.float16), torch.zeros(1, 8, dtype=torch.int32), 3)
    with pytest.raises(ValueError, match="group_size"):
        tob.awq_dequantize(torch.zeros(96, 8, dtype=torch.int32), torch.zeros(2, 64),
                           torch.zeros(2, 8, dtype=torch.int32))
    with pytest.raises(NotImplementedError, match="tma_aligned_scales"):
        tob.per_token_group_quant_fp8(torch.zeros(2, 8), 8, tma_aligned_scales=True)
    with pytest.raises(ValueError, match="divisible"):
        tob.per_token_group_quant_fp8(torch.zeros(2, 9), 8)
    with pytest.raises(TypeError, match="int8"):
        tob.per_token_group_quant_int8(torch.zeros(2, 8), 8, dtype=torch.int16)
    with pytest.raises(ValueError, match="length 2"):
        tob.w8a8_block_int8_matmul(torch.zeros(2, 8, dtype=torch.int8),
                                   torch.zeros(2, 8, dtype=torch.int8), torch.ones(2, 1),
                                   torch.ones(1, 1), [2, 4, 8])
    with pytest.raises(TypeError, match="must be int8"):
        tob.w8a8_block_int8_matmul(torch.zeros(2, 8), torch.zeros(2, 8, dtype=torch.int8),
                                   torch.ones(2, 1), torch.ones(1, 1), [2, 8])
    with pytest.raises(TypeError, match="FP8"):
        tob.w8a8_block_fp8_matmul(torch.zeros(2, 8), torch.zeros(2, 8), torch.ones(2, 1),
                                  torch.ones(1, 1), [2, 8])
    with pytest.raises(ValueError, match="input_scale"):
        tob.apply_w8a8_block_int8_linear(torch.zeros(2, 8), torch.zeros(2, 8, dtype=torch.int8),
                                         [2, 8], torch.ones(1, 1), input_scale=torch.ones(1))
    with pytest.raises(TypeError, match="float32"):
        tob.quantize_per_tensor(torch.zeros(4), torch.ones(1, dtype=torch.float16))
    with pytest.raises(ValueError, match="positive"):
        tob.quantize_per_tensor(torch.zeros(4), torch.zeros(1))
    with pytest.raises(TypeError, match="floating-point"):
        tob.quantize_per_tensor(torch.zeros(4, dtype=torch.int32), torch.ones(1))
    with pytest.raises(TypeError, match="out_dtype"):
        tob.dequantize_per_tensor(torch.zeros(4, dtype=torch.int8), torch.ones(1),
                                  out_dtype=torch.int32)


def test_fp8_dtype_helpers():
    assert tob.is_fp8(torch.float8_e4m3fn)
    assert tob.is_fp8(torch.zeros(1, dtype=torch.float8_e4m3fn))
    assert not tob.is_fp8(torch.float16)
    assert tob.default_fp8_dtype() == torch.float8_e4m3fn
    assert tob.get_fp8_min_max() == (-448.0, 448.0)
    assert tob.get_fp8_min_max(torch.float8_e4m3fnuz) == (-224.0, 224.0)


def test_dropin_module_names():
    import tileops
    import tileops.quant_awq as qa

    assert tileops.awq_gemm is tob.awq_gemm
    assert qa.REVERSE_AWQ_ORDER == (0, 4, 1, 5, 2, 6, 3, 7)
    assert tileops.AWQ_TRITON_SUPPORTED_GROUP_SIZES == [-1, 32, 64, 128]
    for name in ("block_dequant_fp8", "w8a8_triton_block_scaled_mm", "awq_dequantize_triton",
                 "apply_w8a8_block_fp8_linear", "dequantize_per_channel"):
        assert hasattr(tileops, name)


def test_fused_and_gemm_validation_before_compute():
    """The checks of tileops/fused.py:34-64, tileops/blas/gemm.py:41-50 and
    tileops/blas/gemv.py:32-43, raised before any device work (so they hold on CPU tensors
    too)."""
    with pytest.raises(ValueError, match="shape mismatch"):
        tob.silu_and_mul(torch.zeros(2, 3), torch.zeros(2, 4))
    with pytest.raises(TypeError, match="dtype mismatch"):
        tob.gelu_and_mul(torch.zeros(2, 3), torch.zeros(2, 3, dtype=torch.float16))
    with pytest.raises(ValueError, match="out.shape"):
        tob.silu_and_mul(torch.zeros(2, 3), torch.zeros(2, 3), out=torch.zeros(3, 2))
    with pytest.raises(TypeError, match="out.dtype"):
        tob.silu_and_mul(torch.zeros(2, 3), torch.zeros(2, 3),
                         out=torch.zeros(2, 3, dtype=torch.float16))
    with pytest.raises(TypeError, match="CUDA"):
        tob.silu_and_mul(torch.zeros(2, 3), torch.zeros(2, 3))
    with pytest.raises(ValueError, match="2-D"):
        tob.gemm(torch.zeros(3), torch.zeros(3, 4))
    with pytest.raises(ValueError, match="incompatible"):
        tob.mm(torch.zeros(2, 3), torch.zeros(4, 5))
    with pytest.raises(TypeError, match="dtypes must match"):
        tob.gemm(torch.zeros(2, 3), torch.zeros(3, 4, dtype=torch.float16))
    with pytest.raises(TypeError, match="CUDA"):
        tob.gemm(torch.zeros(2, 3), torch.zeros(3, 4))
    # tileops/blas/gemv.py:32-43
    with pytest.raises(ValueError, match="A 2-D and x 1-D"):
        tob.gemv(torch.zeros(2, 3), torch.zeros(2, 3))
    with pytest.raises(ValueError, match="len"):
        tob.mv(torch.zeros(2, 3), torch.zeros(4))
    with pytest.raises(TypeError, match="dtypes must match"):
        tob.gemv(torch.zeros(2, 3), torch.zeros(3, dtype=torch.float16))
    with pytest.raises(ValueError, match="Unsupported dtype"):
        tob.gemv(torch.zeros(2, 3, dtype=torch.int8), torch.zeros(3, dtype=torch.int8))
    with pytest.raises(TypeError, match="CUDA"):
        tob.gemv(torch.zeros(2, 3), torch.zeros(3))


def test_dropin_fused_and_blas_names():
    import tileops
    import tileops.fused as tf

    assert tileops.silu_and_mul is tob.silu_and_mul and tf.gelu_and_mul is tob.gelu_and_mul
    assert tileops.gemm is tob.gemm and tileops.mm is tob.mm
    assert tileops.gemv is tob.gemv and tileops.mv is tob.mv
    from tileops.blas import gemm, gemv, mm, mv
    from tileops.blas.gemv import gemv as gemv2

    assert (gemm, gemv, mm, mv, gemv2) == (tob.gemm, tob.gemv, tob.mm, tob.mv, tob.gemv)


def test_public_signatures_match_the_reference():
    """Every public function of the replaced reference modules exists under the same module
    path of the drop-in package with the same parameter names, kinds and defaults
    (tests/golden/signatures.json, recorded from the reference by make_signatures.py)."""
    import importlib
    import inspect
    import json

    import tileops  # noqa: F401  (installs the module aliases)

    spec = json.loads((Path(__file__).resolve().parent / "golden" / "signatures.json").read_text())
    assert sum(len(v) for v in spec.values()) >= 30
    for mod_name, funcs in spec.items():
        mod = importlib.import_module(mod_name)
        for name, params in funcs.items():
            fn = getattr(mod, name, None)
            assert fn is not None, f"{mod_name}.{name} missing"
            got = []
            for p in inspect.signature(fn).parameters.values():
                d = "" if p.default is inspect.Parameter.empty else f"={p.default!r}"
                got.append(f"{p.name}:{p.kind.name}{d}")
            assert got == params, f"{mod_name}.{name}: {got} != {params}"


def test_argument_errors_match_the_reference():
    """Each invalid call of tests/golden/error_cases.py raises the exception type and message the
    reference raises for it (tests/golden/errors.json, recorded by make_errors.py)."""
    import json

    import tileops  # noqa: F401  (installs the module aliases)
    from tileops import fused, quant, quant_awq, quant_fp8, quant_int8

    golden_dir = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(golden_dir))
    try:
        import error_cases
    finally:
        sys.path.remove(str(golden_dir))
    want = json.loads((golden_dir / "errors.json").read_text())
    got = error_cases.run(error_cases.cases(quant_awq, quant_int8, quant_fp8, quant, fused))
    assert set(got) == set(want)
    for name in want:
        assert got[name] == want[name], f"{name}: {got[name]} != {want[name]}"


def test_interleave_gate_up_is_a_column_permutation():
    """awq_interleave_gate_up reorders whole packed words and scale columns: the dequantised
    interleaved weight is the original's columns in the order gate block j, up block j."""
    import torch

    from oracle import awq as oawq
    from tileops_b200.quant_awq import awq_interleave_gate_up

    gen = torch.Generator().manual_seed(5)
    k, n, g = 256, 96, 64
    w = torch.randint(0, 16, (k, n), generator=gen, dtype=torch.int64)
    z = torch.randint(0, 16, (k // g, n), generator=gen, dtype=torch.int64)
    s = torch.rand(k // g, n, generator=gen).half()
    qw, qz = torch.from_numpy(oawq.pack(w.numpy())), torch.from_numpy(oawq.pack(z.numpy()))
    qw_i, s_i, qz_i = awq_interleave_gate_up(qw, s, qz)
    perm = []
    for j in range(n // 16):
        perm += list(range(8 * j, 8 * j + 8)) + list(range(n // 2 + 8 * j, n // 2 + 8 * j + 8))
    full = oawq.dequant(qw.numpy(), s.float().numpy(), qz.numpy(), "f16")
    inter = oawq.dequant(qw_i.numpy(), s_i.float().numpy(), qz_i.numpy(), "f16")
    assert np.array_equal(inter, full[:, perm])
    with pytest.raises(ValueError):
        awq_interleave_gate_up(qw[:, :1], s[:, :8], qz[:, :1])
