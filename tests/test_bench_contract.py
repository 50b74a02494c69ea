"""The CPU side of bench.py's output contract: the reference arm (the CPU restatement timed on the
host) prints one JSON line with the GPU arm's metric, unit, direction and config, a
`cpu_baseline` describing the sample and an `e2e` object with no host-device bytes; under a
multi-rank launch only rank 0 prints."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    p = _run({}, "--impl", "reference", "--workload", "dense_gemv", "--steps", "2",
             "--warmup", "3")
    assert p.returncode == 0, p.stderr
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    wl = bench.WORKLOADS["dense_gemv"]
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == wl.unit
    assert line["higher_is_better"] is True and line["steps"] == 2 and line["warmup"] == 3
    assert line["config"] == bench.arm_config(wl, 1, 16)
    assert line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == wl.unit and cb["kind"] == "port"
    assert cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": wl.unit, "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_are_silent():
    p = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--impl", "reference",
             "--workload", "dense_gemv", "--steps", "1", "--warmup", "3", "--gpus", "2")
    assert p.returncode == 0, p.stderr
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_every_workload_has_a_config_and_units(name):
    wl = bench.WORKLOADS[name]
    cfg = bench.arm_config(wl, 2, 16)
    assert isinstance(cfg.get("workload"), str) and cfg["workload"]
    assert "model" not in cfg
    assert wl.unit in ("GB/s", "TFLOP/s", "TOPS")
    assert wl.bound in ("hbm", "tensor") and wl.scaling in ("weak", "strong")
    assert wl.launches_per_step >= 1


def test_reference_arm_reports_every_config():
    """The default reference arm also times the CPU restatement of the other configurations, so
    each GPU `workloads` entry has its CPU counterpart."""
    p = _run({}, "--impl", "reference", "--steps", "1", "--warmup", "3")
    assert p.returncode == 0, p.stderr
    line = json.loads([ln for ln in p.stdout.splitlines() if ln.startswith("{")][0])
    subs = line["workloads"]
    assert set(subs) == {key for key, _, _ in bench.SUB_WORKLOADS}
    for key, name, m in bench.SUB_WORKLOADS:
        wl = bench.WORKLOADS[name]
        e = subs[key]
        assert e["value"] > 0 and e["unit"] == wl.unit
        assert e["cpu_baseline"]["kind"] == "port" and e["cpu_baseline"]["cores"] >= 1
        if m is not None:
            assert e["config"]["M"] == m
