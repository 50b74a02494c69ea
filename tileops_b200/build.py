"""Builds libtileops_b200.so in-tree from tileops_b200/csrc/*.cu with nvcc for sm_100a.

Usage: ``python -m tileops_b200.build [--force] [--verbose]``. Objects go to
``tileops_b200/_build/``; the shared library lands next to this file so that it travels
with the source tree. Recompiles a translation unit when it or any header is newer than
its object.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libtileops_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-DTOB_BUILD",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or newest_header > t


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool, ptxas_v: bool) -> tuple[Path, str]:
    cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return src, res.stderr


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    """Compiles every CUDA source and links the shared library; returns its path."""
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources in {CSRC}")
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objs = [BUILD / (s.stem + ".o") for s in sources]
    todo = [(s, o) for s, o in zip(sources, objs) if force or _stale(o, s, newest_header)]
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose, ptxas_v) for s, o in todo]
            for f in cf.as_completed(futs):
                src, log = f.result()
                if ptxas_v and log:
                    print(f"--- {src.name}\n{log}", flush=True)
    if force or todo or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    args = ap.parse_args(argv)
    lib = build(force=args.force, verbose=args.verbose, ptxas_v=args.ptxas_v)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
