"""Concurrent TP-rank saves into one Storage under pool pressure
(tests/storage_reclaim_concurrent.cpp): while every rank allocates and
evicts at once, no allocation may fail for want of memory that another
thread has evicted but not yet released, and every step's blocks must seal
with one owner per rank. Repeated runs, since the race is timing dependent.
CPU only."""

import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


@pytest.fixture(scope="module")
def exe():
    out = ROOT / "tests" / "_build" / "storage_reclaim_concurrent"
    out.parent.mkdir(exist_ok=True)
    srcs = [ROOT / "tests" / "storage_reclaim_concurrent.cpp", CSRC / "storage.cpp", CSRC / "offset_allocator.cpp",
            CSRC / "pinned.cpp"]
    cmd = ["g++", "-O2", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           *map(str, srcs), f"-L{CUDA / 'lib64'}", "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", str(out)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return out


@pytest.mark.parametrize("tp", [4, 8])
def test_concurrent_saves_under_eviction_never_fail_allocation(exe, tp):
    for _ in range(6):
        res = subprocess.run([str(exe), str(tp), "8"], capture_output=True, text=True, timeout=120)
        assert res.returncode == 0, res.stdout + res.stderr
        assert res.stdout.strip().startswith(f"ok tp={tp}"), res.stdout
