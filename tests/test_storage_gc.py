"""Stale inflight blocks (a block that lost a slot to the cached-then-evicted
race of a per-layer save, pegaflow-core/src/lib.rs:604-611) are released
with their pool memory after the age limit, and only they are
(tests/storage_gc.cpp). CPU only."""

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


def test_stale_inflight_blocks_are_released():
    exe = ROOT / "tests" / "_build" / "storage_gc"
    exe.parent.mkdir(exist_ok=True)
    srcs = [ROOT / "tests" / "storage_gc.cpp", CSRC / "storage.cpp", CSRC / "offset_allocator.cpp",
            CSRC / "pinned.cpp"]
    cmd = ["g++", "-O1", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           *map(str, srcs), f"-L{CUDA / 'lib64'}", "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip().splitlines()[-1] == "ok"
