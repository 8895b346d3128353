"""Concurrent TP-rank slot inserts into one Storage end in the same state as
inserting the ranks one after another (tests/storage_tp_concurrent.cpp): the
inflight map is sharded so that ranks proceed in parallel, and this checks
that the sharding loses or duplicates nothing. CPU only."""

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


def test_concurrent_rank_inserts_match_serial_inserts():
    exe = ROOT / "tests" / "_build" / "storage_tp_concurrent"
    exe.parent.mkdir(exist_ok=True)
    srcs = [ROOT / "tests" / "storage_tp_concurrent.cpp", CSRC / "storage.cpp", CSRC / "offset_allocator.cpp",
            CSRC / "pinned.cpp"]
    cmd = ["g++", "-O1", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           *map(str, srcs), f"-L{CUDA / 'lib64'}", "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe), "200"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    line = out.stdout.strip().splitlines()[-1]
    counts = dict(kv.split("=") for kv in line.split()[1:])
    assert line.startswith("ok") and int(counts["sealed"]) > 1000, line
