"""The staging-chunk cutter on the CPU (tests/chunks_test.cpp): every chunk
fits its staging slot with an aligned start, the chunks tile the plan, each
tile's bytes lie inside its chunk, the growth limits hold, and the benchmark's
documented schedules come out as stated."""

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


def test_chunk_cutter_invariants_and_schedules():
    exe = ROOT / "tests" / "_build" / "chunks_test"
    exe.parent.mkdir(exist_ok=True)
    cmd = ["g++", "-O1", "-std=c++17", f"-I{CSRC}", f"-I{CUDA / 'include'}", str(ROOT / "tests" / "chunks_test.cpp"),
           str(CSRC / "chunks.cpp"), "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip().splitlines()[-1].startswith("ok")
