"""Storage over several pools (the engine's numa_pools modes): allocations
go to the pool they name, reclaim for a pool evicts only blocks held there,
usage sums the pools, and a pool placed on a NUMA node lands there
(tests/storage_pools.cpp). CPU only."""

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


def test_pools_route_and_reclaim_separately():
    exe = ROOT / "tests" / "_build" / "storage_pools"
    exe.parent.mkdir(exist_ok=True)
    srcs = [ROOT / "tests" / "storage_pools.cpp", CSRC / "storage.cpp", CSRC / "offset_allocator.cpp",
            CSRC / "pinned.cpp"]
    cmd = ["g++", "-O1", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           *map(str, srcs), f"-L{CUDA / 'lib64'}", "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip().splitlines()[-1] == "ok"


def test_engine_rejects_unknown_numa_mode():
    import pytest

    from pegaflow_b200 import PegaEngine

    with pytest.raises(ValueError, match="numa_pools"):
        PegaEngine(1 << 20, pool_kind="host", numa_pools="socket")
    PegaEngine(1 << 20, pool_kind="host", numa_pools="node").close()  # host pools stay single
