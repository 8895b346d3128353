"""The C ABI library loads and exports every entry point include/pegaflow.h declares."""

import re
from pathlib import Path

HEADER = Path(__file__).resolve().parent.parent / "include" / "pegaflow.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(pf_[a-z0-9_]+)\s*\(", text))


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"pf_save_blocks", "pf_load_blocks", "pf_engine_batch_load_kv_blocks", "pf_load_state_create"} <= names


def test_library_exports_every_declared_symbol(native):
    missing = [n for n in sorted(declared_functions()) if not hasattr(native.lib, n)]
    assert not missing, f"symbols declared in pegaflow.h but not exported: {missing}"


def test_binding_covers_header(native):
    assert declared_functions() == set(native.SYMBOLS)


def test_abi_version(native):
    assert native.lib.pf_abi_version() == 3


def test_library_is_sm100a_build(native):
    """The library embeds sm_100a device code (checked by the build, not by
    inspecting the binary): the build flags pin -gencode arch=compute_100a."""
    from pegaflow_b200 import build

    assert ["-gencode", "arch=compute_100a,code=sm_100a"] == build.ARCH
