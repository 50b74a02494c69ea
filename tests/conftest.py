"""Shared test configuration: the ``gpu`` marker, golden-fixture loading and helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"

_TORCH_DTYPES = {
    "float32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "float8_e4m3fn": torch.float8_e4m3fn,
    "float8_e4m3fnuz": torch.float8_e4m3fnuz,
    "int8": torch.int8,
    "int32": torch.int32,
    "int64": torch.int64,
}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) and libtileops_b200.so")


class GoldenCase(dict):
    """Fields of one golden case; ``tensor(name, device)`` rebuilds the original dtype."""

    def tensor(self, field: str, device="cpu") -> torch.Tensor:
        arr = self[field]
        dt = self.get(field + ".dtype")
        if dt is None:
            return torch.from_numpy(np.array(arr)).to(device)
        dt = _TORCH_DTYPES[str(dt)]
        if dt in (torch.float8_e4m3fn, torch.float8_e4m3fnuz):
            return torch.from_numpy(np.array(arr, dtype=np.uint8)).view(dt).to(device)
        if dt == torch.bfloat16:
            # bf16 values are stored as their exact fp32 values: keep the top 16 bits, so a NaN
            # keeps its sign (torch's vectorised fp32 -> bf16 cast would rewrite it)
            bits = (np.array(arr, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
            return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)
        return torch.from_numpy(np.array(arr)).to(dt).to(device)

    def dtype_name(self, field: str) -> str:
        return {"float32": "f32", "float16": "f16", "bfloat16": "bf16"}[str(self[field + ".dtype"])]


def load_golden(name: str) -> dict[str, GoldenCase]:
    data = np.load(GOLDEN / name, allow_pickle=False)
    cases: dict[str, GoldenCase] = {}
    for key in data.files:
        case, field = key.split("/", 1)
        cases.setdefault(case, GoldenCase())[field] = data[key]
    return cases


@pytest.fixture(scope="session")
def golden():
    cache: dict[str, dict[str, GoldenCase]] = {}

    def get(name: str) -> dict[str, GoldenCase]:
        if name not in cache:
            cache[name] = load_golden(name)
        return cache[name]

    return get


@pytest.fixture(scope="session")
def cuda():
    """The device for GPU tests; fails (not skips) when the library cannot run there."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a host without CUDA")
    import tileops_b200._lib as lib

    lib.load()
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _device_error_word_clear(request):
    """After every GPU test: no kernel may have left a bounded-wait timeout behind."""
    yield
    if request.node.get_closest_marker("gpu") is None or not torch.cuda.is_available():
        return
    import tileops_b200._lib as lib

    assert lib.device_error_word(clear=True) == 0, "a kernel's bounded wait expired"
