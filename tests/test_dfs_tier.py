"""Packed-file tier (the reference's DFS offload, seal_offload.rs) on the CPU:
the tier's logic and file format through tests/dfs_tier_test.cpp, the
record encoding against the oracle's restatement, and the engine-level API
on a plain-memory engine."""

import json
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


def test_tier_write_prefetch_restart_quota(tmp_path):
    exe = ROOT / "tests" / "_build" / "dfs_tier_test"
    exe.parent.mkdir(exist_ok=True)
    srcs = [ROOT / "tests" / "dfs_tier_test.cpp", CSRC / "dfs_tier.cpp", CSRC / "storage.cpp",
            CSRC / "offset_allocator.cpp", CSRC / "pinned.cpp"]
    cmd = ["g++", "-O1", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           *map(str, srcs), f"-L{CUDA / 'lib64'}", "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    root = tmp_path / "dfs"
    root.mkdir()
    out = subprocess.run([str(exe), str(root)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stdout + out.stderr


def test_record_encoding_matches_oracle():
    """serde_json's compact encoding of BlockMeta, restated by the oracle,
    for the layouts a block can hold (split and contiguous slots)."""
    from oracle import oracle

    data, metas = oracle.dfs_pack([[(b"K" * 4, b"V" * 4), (b"C" * 6, None)],
                                   [(b"k" * 4, b"v" * 4), (b"c" * 6, None)]], "f.bin")
    assert data == b"KKKKVVVVCCCCCC" + b"kkkkvvvvcccccc"
    assert metas[1] == ('{"file":"f.bin","offset":14,"slots":[{"is_split":true,"size":8},'
                        '{"is_split":false,"size":6}],"total_slots":2}')
    assert json.loads(metas[0])["offset"] == 0
    assert oracle.dfs_file_meta([b"\x00\xff"], 28) == '{"blocks":["00ff"],"size":28}'


def test_engine_query_prefetch_api(native, tmp_path):
    from pegaflow_b200 import PegaEngine

    # Tier off: the plain prefix count, reported as ready.
    e = PegaEngine(1 << 20, pool_kind="host")
    e.register_context_layer("i", "ns", 0, "L0", 0x7000_0000, 2 * 16 * 4096, 16, 4096, 16 * 4096, 2, 0, 1, 1)
    assert e.query_prefetch("i", [b"a", b"b"]) == {"hit_blocks": 0, "prefetch_state": "ready",
                                                   "loading_blocks": 0, "missing_blocks": 0}
    with pytest.raises(RuntimeError, match="packed-file tier is off"):
        e.dfs_stats()
    e.close()
    # Tier on, nothing written yet: the first block is nowhere.
    e = PegaEngine(1 << 20, pool_kind="host", dfs_root=str(tmp_path / "dfs"), dfs_max_pack_size=8)
    e.register_context_layer("i", "ns", 0, "L0", 0x7000_0000, 2 * 16 * 4096, 16, 4096, 16 * 4096, 2, 0, 1, 1)
    q = e.query_prefetch("i", [b"a", b"b"])
    assert q == {"hit_blocks": 0, "prefetch_state": "partial_miss", "loading_blocks": 0, "missing_blocks": 2}
    assert e.dfs_flush(5.0)
    st = e.dfs_stats()
    assert st["files"] == 0 and st["written_blocks"] == 0
    e.dfs_check_quota()
    e.close()
    assert (tmp_path / "dfs").is_dir()
