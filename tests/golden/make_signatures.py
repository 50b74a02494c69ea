"""Records the public signatures of the reference's modules that this library replaces
(parameter names, kinds and defaults) in signatures.json, so that a CPU test can check the
drop-in API without the reference checkout. Run from the repository root:

    python tests/golden/make_signatures.py

The reference is imported from the checkout named by the required TILEOPS_REF variable."""

from __future__ import annotations

import importlib
import inspect
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
if not os.environ.get("TILEOPS_REF"):
    sys.exit("set TILEOPS_REF to the TileOps checkout to record")
REF = Path(os.environ["TILEOPS_REF"])
sys.path.insert(0, str(REF))

# module -> the public functions this library provides from it (None: every public function
# the module defines)
MODULES = {
    "tileops.quant_awq": None,
    "tileops.quant_int8": None,
    "tileops.quant_fp8": None,
    "tileops.quant": None,
    "tileops.fused": ["silu_and_mul", "gelu_and_mul"],
    "tileops.blas.gemm": ["gemm", "mm"],
    "tileops.blas.gemv": ["gemv", "mv"],
}


def describe(fn) -> list[str]:
    """One "name:KIND=default" string per parameter ("name:KIND" without a default)."""
    out = []
    for p in inspect.signature(fn).parameters.values():
        d = "" if p.default is inspect.Parameter.empty else f"={p.default!r}"
        out.append(f"{p.name}:{p.kind.name}{d}")
    return out


def main() -> None:
    out = {}
    for mod_name, names in MODULES.items():
        mod = importlib.import_module(mod_name)
        assert Path(mod.__file__).resolve().is_relative_to(REF.resolve()), mod.__file__
        if names is None:
            names = sorted(n for n, f in inspect.getmembers(mod, inspect.isfunction)
                           if f.__module__ == mod.__name__ and not n.startswith("_"))
        out[mod_name] = {n: describe(getattr(mod, n)) for n in names}
    (HERE / "signatures.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print("signatures.json:", sum(len(v) for v in out.values()), "functions")


if __name__ == "__main__":
    main()
