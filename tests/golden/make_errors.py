"""Records the exception type and message the reference raises for each invalid call of
error_cases.py in errors.json. Run from the repository root:

    python tests/golden/make_errors.py

The reference is imported from the checkout named by the required TILEOPS_REF variable."""

from __future__ import annotations

import importlib
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
if not os.environ.get("TILEOPS_REF"):
    sys.exit("set TILEOPS_REF to the TileOps checkout to record")
REF = Path(os.environ["TILEOPS_REF"])
sys.path.insert(0, str(REF))
sys.path.insert(1, str(HERE))

import error_cases  # noqa: E402


def main() -> None:
    mods = [importlib.import_module(f"tileops.{m}")
            for m in ("quant_awq", "quant_int8", "quant_fp8", "quant", "fused")]
    for m in mods:
        assert Path(m.__file__).resolve().is_relative_to(REF.resolve()), m.__file__
    out = error_cases.run(error_cases.cases(*mods))
    (HERE / "errors.json").write_text(json.dumps(out, indent=1, sort_keys=True,
                                                 ensure_ascii=False) + "\n")
    print("errors.json:", len(out), "cases")


if __name__ == "__main__":
    main()
