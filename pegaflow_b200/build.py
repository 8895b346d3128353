"""Builds libpegaflow_b200.so (sm_100a kernels + C++ engine + C ABI) in-tree.

Every translation unit is compiled by nvcc for sm_100a only; the shared
library lands next to this file so it travels with the source tree.
Run: python -m pegaflow_b200.build [--force]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libpegaflow_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-Wall,-Wno-unused-function",
    f"-I{ROOT / 'include'}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build pegaflow_b200")


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library if any source or header changed."""
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    headers = _headers()
    jobs = []
    objs = []
    for src in _sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            jobs.append([cc, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)])

    def run(cmd: list[str]) -> None:
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        if verbose and res.stderr.strip():
            print(res.stderr, flush=True)

    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static", "-lrt", "-lpthread"]
        run(cmd)
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
