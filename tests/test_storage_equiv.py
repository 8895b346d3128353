"""The engine's hash-major slot insert (Storage::insert_slots_multi, used when
every layer of a save carries the same hash list) against the per-layer
insert it replaces, on random pre-states: identical cache contents and LRU
order, inflight slots, admission counters and errors (tests/storage_equiv.cpp).
CPU only."""

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


def test_multi_slot_insert_matches_per_layer_insert():
    exe = ROOT / "tests" / "_build" / "storage_equiv"
    exe.parent.mkdir(exist_ok=True)
    srcs = [ROOT / "tests" / "storage_equiv.cpp", CSRC / "storage.cpp", CSRC / "offset_allocator.cpp",
            CSRC / "pinned.cpp"]
    cmd = ["g++", "-O1", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           *map(str, srcs), f"-L{CUDA / 'lib64'}", "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe), "20000"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    line = out.stdout.strip().splitlines()[-1]
    assert line.startswith("ok"), line
    counts = dict(kv.split("=") for kv in line.split()[1:])
    # The random pre-states must reach every branch: seals, refusals, errors.
    assert int(counts["seals"]) > 1000 and int(counts["refusals"]) > 50 and int(counts["errors"]) > 100, line
