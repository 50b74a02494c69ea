"""CPU oracle for the TileOps quantized-linear path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's arithmetic (llongmarch/TileOps, files
tileops/quant_awq.py, tileops/quant_int8.py, tileops/quant_fp8.py, tileops/quant.py),
each function citing the reference lines it follows. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may import it,
and only as the checker or the timed CPU baseline; the product (``tileops_b200``) never
calls it and has no CPU path.

Pinning: every function here is checked against golden vectors produced by running the
reference itself on seeded inputs (``tests/golden/make_golden.py`` ->
``tests/golden/*.npz``, asserted by ``tests/test_oracle_golden.py``), and against the
known-answer vectors of the reference's own tests (tests/awq.py, tests/int8_utils.py,
tests/fp8.py, tests/quant.py).
"""

from . import awq, fp8, int8, numerics, sym  # noqa: F401
