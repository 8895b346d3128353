"""Byte parity of the library's own transfer plans on the CPU
(tests/plan_emulator.cpp): plan_save / plan_load and the staging-chunk cutter
are replayed on host arrays with the copy kernel's tile addressing and the
copy-engine runs, and the pool and restored bytes must equal the C oracle's
restatement of the reference's copies; peer-copy plans (plan_p2p) must give
copy identity. It caught a save bug the GPU tests
missed by timing: a chunk whose first byte is not 256-byte aligned had its
copy start at the aligned slot base, so stale slot bytes could overwrite the
previous chunk's last bytes in the pool."""

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


def test_plans_replayed_on_the_cpu_match_the_oracle():
    build = ROOT / "tests" / "_build"
    build.mkdir(exist_ok=True)
    obj = build / "pf_oracle_emu.o"
    subprocess.run(["gcc", "-O1", "-c", str(ROOT / "oracle" / "pf_oracle.c"), "-o", str(obj)], check=True,
                   capture_output=True, text=True)
    exe = build / "plan_emulator"
    cmd = ["g++", "-O1", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           str(ROOT / "tests" / "plan_emulator.cpp"), str(CSRC / "plan_build.cpp"), str(CSRC / "chunks.cpp"), str(obj),
           f"-L{CUDA / 'lib64'}", "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe), "3000"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    line = out.stdout.strip().splitlines()[-1]
    assert line.startswith("ok"), line
    counts = dict(kv.split("=") for kv in line.split()[1:])
    assert int(counts["loads"]) > 2500 and int(counts["serial"]) > 100 and int(counts["peers"]) > 5000, line
    assert int(counts["within"]) == 3000, line
