"""Drop-in name for code written against the reference: ``from tileops import awq_gemm`` and
``import tileops.quant_awq`` resolve to the sm_100a implementation in :mod:`tileops_b200`.
Only the quantized-linear modules, the gated activations of ``tileops.fused``
(``silu_and_mul``, ``gelu_and_mul``) and the dense ``gemm`` / ``mm`` / ``gemv`` / ``mv``
comparators are provided (also as ``tileops.blas``); the rest of the reference package (other
elementwise ops, norms, attention, other BLAS, Metal backends) is not part of this library."""

import sys as _sys

import tileops_b200 as _impl
from tileops_b200 import *  # noqa: F401,F403
from tileops_b200 import __all__  # noqa: F401
from tileops_b200 import blas, fused, quant, quant_awq, quant_fp8, quant_int8  # noqa: F401

for _name in ("blas", "fused", "quant", "quant_awq", "quant_fp8", "quant_int8"):
    _sys.modules[f"{__name__}.{_name}"] = getattr(_impl, _name)
# the reference's tileops/blas/gemm.py and gemv.py define these names; both map to one module
_sys.modules[f"{__name__}.blas.gemm"] = _impl.blas
_sys.modules[f"{__name__}.blas.gemv"] = _impl.blas
