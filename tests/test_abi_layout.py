"""The ctypes mirrors in pegaflow_b200/_native.py match the structs of
include/pegaflow.h byte for byte: a C program built against the header prints
each struct's size and the offset of every field the mirror declares, and
both must equal what ctypes computes. A field added on one side only (or in
another order) fails here instead of corrupting memory at run time. CPU only."""

import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent

PAIRS = {
    "pf_layer_desc": "LayerDesc",
    "pf_executor_config": "ExecutorConfig",
    "pf_save_layer": "SaveLayer",
    "pf_load_layer": "LoadLayer",
    "pf_executor_stats": "ExecutorStats",
    "pf_p2p_layer": "P2PLayer",
    "pf_engine_config": "EngineConfig",
    "pf_bytes": "Bytes",
    "pf_prefetch_status": "PrefetchStatus",
    "pf_dfs_stats": "DfsStats",
    "pf_save_entry": "SaveEntry",
    "pf_engine_metrics": "EngineMetrics",
}


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    from pegaflow_b200 import _native as N

    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "pegaflow.h"', "int main(void) {"]
    for c_name, py_name in PAIRS.items():
        cls = getattr(N, py_name)
        lines.append(f'  printf("{c_name} size %zu\\n", sizeof({c_name}));')
        for field, _ in cls._fields_:
            lines.append(f'  printf("{c_name} {field} %zu\\n", offsetof({c_name}, {field}));')
    lines += ["  return 0;", "}"]
    d = tmp_path_factory.mktemp("abi")
    src, exe = d / "layout.c", d / "layout"
    src.write_text("\n".join(lines) + "\n")
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True,
                   capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    table = {}
    for line in out.splitlines():
        struct, field, value = line.split()
        table[(struct, field)] = int(value)
    return table


@pytest.mark.parametrize("c_name", sorted(PAIRS))
def test_ctypes_mirror_matches_header(c_layout, c_name):
    from ctypes import sizeof

    from pegaflow_b200 import _native as N

    cls = getattr(N, PAIRS[c_name])
    assert sizeof(cls) == c_layout[(c_name, "size")], c_name
    for field, _ in cls._fields_:
        assert getattr(cls, field).offset == c_layout[(c_name, field)], (c_name, field)
