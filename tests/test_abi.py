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
    assert native.lib.pf_abi_version() == 4 == native.ABI_VERSION


def test_config_defaults(native):
    """Library defaults: the reference's 30 GiB write-combined pool with TinyLFU
    admission (lib.rs:56, pinned_mem.rs:159, storage.rs:91), one pool (no NUMA
    split), 2 x 1 GiB staging slots per lane, the copy kernel chosen per
    transfer (bulk copies where they apply)."""
    from ctypes import byref

    e = native.EngineConfig()
    native.lib.pf_engine_config_default(byref(e))
    assert (e.pool_bytes, e.write_combined, e.enable_lfu_admission, e.numa_pools) == (30 << 30, 1, 1, 0)
    assert (e.pre_evict_enabled, e.pre_evict_threshold_bytes, e.pre_evict_target_bytes) == (0, 5 << 30, 8 << 30)
    x = native.ExecutorConfig()
    native.lib.pf_executor_config_default(byref(x))
    assert (x.staging_chunk_bytes, x.staging_slots, x.first_chunk_bytes) == (1 << 30, 2, 256 << 20)
    assert x.copy_kernel == native.PF_COPY_KERNEL_AUTO


def test_library_is_sm100a_build(native):
    """The library embeds sm_100a device code (checked by the build, not by
    inspecting the binary): the build flags pin -gencode arch=compute_100a."""
    from pegaflow_b200 import build

    assert ["-gencode", "arch=compute_100a,code=sm_100a"] == build.ARCH


def test_noalloc_argument_errors_need_no_gpu(native):
    """The no-allocation save refuses a null layer array before touching CUDA,
    and on a host without a GPU an empty save fails with the CUDA-init code
    (lib.rs:58-67's CudaInit variant) instead of crashing."""
    import torch

    rc = native.lib.pf_save_blocks_noalloc(0, None, 1, None)
    assert rc == native.PF_ERR_INVALID_ARGUMENT
    assert "null layers" in native.lib.pf_last_error().decode()
    if not torch.cuda.is_available():
        assert native.lib.pf_save_blocks_noalloc(0, None, 0, None) == native.PF_ERR_CUDA_INIT
        assert native.lib.pf_save_blocks_noalloc(-1, None, 0, None) == native.PF_ERR_CUDA_INIT
