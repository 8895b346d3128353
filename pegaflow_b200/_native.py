"""ctypes binding of include/pegaflow.h (the library's C ABI).

The shared library is built in-tree by ``pegaflow_b200.build``. Importing this
module never falls back to anything else: if the library is missing or does
not load, the import fails with the reason.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import (
    POINTER,
    Structure,
    c_char_p,
    c_double,
    c_int,
    c_int32,
    c_int64,
    c_uint8,
    c_uint32,
    c_uint64,
    c_void_p,
)
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpegaflow_b200.so"
ABI_VERSION = 4  # PF_ABI_VERSION the structs below follow

PF_OK = 0
PF_ERR_INSTANCE_MISSING = 1
PF_ERR_WORKER_MISSING = 2
PF_ERR_INVALID_ARGUMENT = 3
PF_ERR_CUDA_INIT = 4
PF_ERR_STORAGE = 5
PF_ERR_POISONED = 6
PF_ERR_TOPOLOGY_MISMATCH = 7
PF_ERR_LOAD_STATE = 8
PF_ERR_TIMEOUT = 9
PF_ERR_NO_SPACE = 10

PF_COPY_KERNEL_AUTO = 0
PF_COPY_KERNEL_REGISTERS = 1
PF_COPY_KERNEL_BULK = 2

PF_MODE_AUTO = 0
PF_MODE_STAGED = 1
PF_MODE_DIRECT = 2

PF_ALLOCATOR_AUTO_UNIT = 2**64 - 1

PF_POOL_PINNED = 0
PF_POOL_HOST = 1


class LayerDesc(Structure):
    _fields_ = [
        ("data_ptr", c_uint64),
        ("size_bytes", c_uint64),
        ("num_blocks", c_uint64),
        ("bytes_per_block", c_uint64),
        ("kv_stride_bytes", c_uint64),
        ("segments", c_uint64),
    ]


class ExecutorConfig(Structure):
    _fields_ = [
        ("staging_chunk_bytes", c_uint64),
        ("staging_slots", c_uint32),
        ("save_mode", c_uint32),
        ("load_mode", c_uint32),
        ("ctas_per_sm", c_uint32),
        ("copy_streams", c_uint32),
        ("cache_streaming", c_uint32),
        ("copy_kernel", c_uint32),
        ("first_chunk_bytes", c_uint64),
    ]


class SaveLayer(Structure):
    _fields_ = [
        ("layer", LayerDesc),
        ("block_idx", POINTER(c_int64)),
        ("n", c_uint64),
        ("k_dst", c_void_p),
        ("v_dst", c_void_p),
    ]


class LoadLayer(Structure):
    _fields_ = [
        ("layer", LayerDesc),
        ("block_idx", POINTER(c_int64)),
        ("n", c_uint64),
        ("k_src", POINTER(c_void_p)),
        ("v_src", POINTER(c_void_p)),
    ]


class ExecutorStats(Structure):
    _fields_ = [
        ("kernel_launches", c_uint64),
        ("copy_calls", c_uint64),
        ("bytes_saved", c_uint64),
        ("bytes_loaded", c_uint64),
        ("kernel_bytes", c_uint64),
        ("kernel_ms", c_double),
        ("timed_launches", c_uint64),
        ("bytes_p2p", c_uint64),
        ("host_ms", c_double),
        ("kernel_body_ms", c_double),
        ("body_launches", c_uint64),
    ]


class P2PLayer(Structure):
    _fields_ = [
        ("src", LayerDesc),
        ("dst", LayerDesc),
        ("src_idx", POINTER(c_int64)),
        ("dst_idx", POINTER(c_int64)),
        ("n", c_uint64),
    ]


class EngineConfig(Structure):
    _fields_ = [
        ("pool_bytes", c_uint64),
        ("use_hugepages", c_int32),
        ("write_combined", c_int32),
        ("enable_lfu_admission", c_int32),
        ("pool_kind", c_int32),
        ("hint_value_size_bytes", c_uint64),
        ("pre_evict_enabled", c_int32),
        ("numa_pools", c_int32),
        ("pre_evict_threshold_bytes", c_uint64),
        ("pre_evict_target_bytes", c_uint64),
        ("pre_evict_interval_ms", c_uint64),
        ("executor", ExecutorConfig),
        ("dfs_root", c_char_p),
        ("dfs_quota_bytes", c_uint64),
        ("dfs_scan_interval_ms", c_uint64),
        ("dfs_max_pack_size", c_uint32),
        ("reserved1", c_uint32),
    ]


class Bytes(Structure):
    _fields_ = [("data", POINTER(c_uint8)), ("len", c_uint64)]


class PrefetchStatus(Structure):
    _fields_ = [
        ("state", c_uint32),
        ("reserved", c_uint32),
        ("hit_blocks", c_uint64),
        ("loading_blocks", c_uint64),
        ("missing_blocks", c_uint64),
    ]


class DfsStats(Structure):
    _fields_ = [(name, c_uint64) for name in (
        "files", "blocks", "usage_bytes", "written_files", "written_blocks", "write_failures",
        "prefetched_blocks", "prefetch_failures", "evicted_files")]


class SaveEntry(Structure):
    _fields_ = [
        ("layer_name", c_char_p),
        ("block_ids", POINTER(c_int32)),
        ("n_ids", c_uint64),
        ("block_hashes", POINTER(Bytes)),
        ("n_hashes", c_uint64),
    ]


class EngineMetrics(Structure):
    _fields_ = [
        ("save_bytes", c_uint64),
        ("save_calls", c_uint64),
        ("save_ms", c_double),
        ("load_bytes", c_uint64),
        ("load_calls", c_uint64),
        ("load_ms", c_double),
        ("load_failures", c_uint64),
        ("cache_block_hits", c_uint64),
        ("cache_block_misses", c_uint64),
        ("cache_block_insertions", c_uint64),
        ("cache_block_admission_rejections", c_uint64),
        ("cache_block_evictions", c_uint64),
        ("pool_alloc_failures", c_uint64),
        ("inflight_blocks", c_uint64),
        ("cached_blocks", c_uint64),
        ("save_plan_ms", c_double),
        ("save_transfer_ms", c_double),
        ("save_insert_ms", c_double),
        ("inflight_dropped", c_uint64),
        ("load_lookup_ms", c_double),
        ("load_queue_ms", c_double),
        ("load_setup_ms", c_double),
        ("load_transfer_ms", c_double),
        ("load_first_layer_ms", c_double),
    ]


# name -> (restype, argtypes)
_SIGNATURES = {
    "pf_last_error": (c_char_p, []),
    "pf_abi_version": (c_int, []),
    "pf_device_count": (c_int, []),
    "pf_layer_validate": (c_int, [POINTER(LayerDesc), c_char_p]),
    "pf_segment_offset": (c_int, [POINTER(LayerDesc), c_uint64, c_uint64, POINTER(c_uint64)]),
    "pf_executor_config_default": (None, [POINTER(ExecutorConfig)]),
    "pf_executor_create": (c_int, [c_int32, POINTER(ExecutorConfig), POINTER(c_void_p)]),
    "pf_executor_destroy": (None, [c_void_p]),
    "pf_save_blocks": (c_int, [c_void_p, POINTER(SaveLayer), c_uint64]),
    "pf_load_blocks": (c_int, [c_void_p, POINTER(LoadLayer), c_uint64]),
    "pf_save_blocks_async": (c_int, [c_void_p, POINTER(SaveLayer), c_uint64, c_void_p]),
    "pf_load_blocks_async": (c_int, [c_void_p, POINTER(LoadLayer), c_uint64, c_void_p, c_void_p]),
    "pf_save_blocks_noalloc": (c_int, [c_int32, POINTER(SaveLayer), c_uint64, c_void_p]),
    "pf_p2p_transfer": (c_int, [c_void_p, c_int32, c_int, POINTER(P2PLayer), c_uint64, c_void_p]),
    "pf_executor_stats_get": (c_int, [c_void_p, POINTER(ExecutorStats)]),
    "pf_executor_stats_reset": (c_int, [c_void_p]),
    "pf_executor_set_timing": (c_int, [c_void_p, c_int]),
    "pf_executor_debug_stall_tile": (c_int, [c_void_p, c_uint64]),
    "pf_refcopy_save": (c_int, [c_int32, POINTER(SaveLayer), c_uint64]),
    "pf_refcopy_load": (c_int, [c_int32, POINTER(LoadLayer), c_uint64, POINTER(c_uint64)]),
    "pf_pinned_alloc": (c_int, [c_uint64, c_int, POINTER(c_void_p)]),
    "pf_pinned_free": (c_int, [c_void_p]),
    "pf_allocator_create": (c_int, [c_uint64, c_uint64, c_uint32, POINTER(c_void_p)]),
    "pf_allocator_destroy": (None, [c_void_p]),
    "pf_allocator_alloc": (c_int, [c_void_p, c_uint64, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint32)]),
    "pf_allocator_free": (None, [c_void_p, c_uint32]),
    "pf_allocator_report": (
        None,
        [c_void_p, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)],
    ),
    "pf_load_state_create": (c_int, [POINTER(c_void_p)]),
    "pf_load_state_attach": (c_int, [c_char_p, POINTER(c_void_p)]),
    "pf_load_state_create_layers": (c_int, [c_uint32, POINTER(c_void_p)]),
    "pf_load_state_layer_count": (c_uint32, [c_void_p]),
    "pf_load_state_layer_get": (c_int64, [c_void_p, c_uint32]),
    "pf_load_state_name": (c_char_p, [c_void_p]),
    "pf_load_state_get": (c_int64, [c_void_p]),
    "pf_load_state_set_completed": (None, [c_void_p]),
    "pf_load_state_set_error": (None, [c_void_p]),
    "pf_load_state_close": (None, [c_void_p]),
    "pf_engine_config_default": (None, [POINTER(EngineConfig)]),
    "pf_engine_create": (c_int, [POINTER(EngineConfig), POINTER(c_void_p)]),
    "pf_engine_destroy": (None, [c_void_p]),
    "pf_engine_register_context_layer": (
        c_int,
        [c_void_p, c_char_p, c_char_p, c_int32, c_char_p]
        + [c_uint64] * 6
        + [c_uint64, c_uint64, c_uint64],
    ),
    "pf_engine_unregister_instance": (c_int, [c_void_p, c_char_p]),
    "pf_engine_batch_save_kv_blocks": (c_int, [c_void_p, c_char_p, c_uint64, c_int32, POINTER(SaveEntry), c_uint64]),
    "pf_engine_save_kv_blocks": (
        c_int,
        [c_void_p, c_char_p, c_uint64, c_int32, c_char_p, POINTER(c_int32), POINTER(Bytes), c_uint64],
    ),
    "pf_engine_count_prefix_hit_blocks": (c_int, [c_void_p, c_char_p, POINTER(Bytes), c_uint64, POINTER(c_uint64)]),
    "pf_engine_query_prefetch": (c_int, [c_void_p, c_char_p, POINTER(Bytes), c_uint64, POINTER(PrefetchStatus)]),
    "pf_engine_dfs_stats": (c_int, [c_void_p, POINTER(DfsStats)]),
    "pf_engine_dfs_flush": (c_int, [c_void_p, c_double, POINTER(c_int)]),
    "pf_engine_dfs_check_quota": (c_int, [c_void_p]),
    "pf_engine_batch_load_kv_blocks": (
        c_int,
        [
            c_void_p,
            c_char_p,
            c_uint64,
            c_int32,
            c_char_p,
            POINTER(c_char_p),
            c_uint64,
            POINTER(c_int32),
            POINTER(Bytes),
            c_uint64,
        ],
    ),
    "pf_engine_wait_loads": (c_int, [c_void_p, c_int32, c_double]),
    "pf_engine_save_request": (c_int, [c_void_p, c_char_p, c_uint64]),
    "pf_engine_load_request": (c_int, [c_void_p, c_char_p, c_uint64]),
    "pf_request_instance_id": (c_int, [c_char_p, c_uint64, c_char_p, c_uint64, POINTER(c_uint64)]),
    "pf_engine_pool_usage": (c_int, [c_void_p, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)]),
    "pf_engine_slot_info": (
        c_int,
        [c_void_p, c_char_p, POINTER(c_uint8), c_uint64, c_uint64, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)],
    ),
    "pf_engine_metrics_get": (c_int, [c_void_p, POINTER(EngineMetrics)]),
    "pf_engine_executor": (c_int, [c_void_p, c_int32, POINTER(c_void_p)]),
}

SYMBOLS = tuple(_SIGNATURES)


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m pegaflow_b200.build` (nvcc, sm_100a)"
        )
    lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_GLOBAL", 0))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.pf_abi_version() != ABI_VERSION:  # the structs above would not match
        raise ImportError(f"{LIB_PATH} has ABI {lib.pf_abi_version()}, these bindings need {ABI_VERSION}: "
                          "rebuild it with `python -m pegaflow_b200.build`")
    return lib


lib = _load()


class PegaError(RuntimeError):
    """A failed C ABI call; ``code`` is the pf_status value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def check(rc: int) -> None:
    if rc != PF_OK:
        msg = lib.pf_last_error()
        raise PegaError(rc, msg.decode("utf-8", "replace") if msg else f"pf_status {rc}")


def bytes_array(items):
    """A pf_bytes[] over a sequence of bytes-like objects, built without a
    per-item ctypes object: the items are joined into one buffer and the
    (pointer, length) pairs are computed with numpy. Returns (pointer,
    keepalive); the keepalive must outlive the C call."""
    import numpy as np

    n = len(items)
    if n == 0:
        empty = (Bytes * 1)()
        return ctypes.cast(empty, POINTER(Bytes)), empty
    items = [x if isinstance(x, bytes) else bytes(x) for x in items]
    blob = b"".join(items)
    lens = np.fromiter(map(len, items), dtype=np.uint64, count=n)
    buf = np.frombuffer(blob, dtype=np.uint8) if blob else np.zeros(1, np.uint8)
    pairs = np.empty((n, 2), dtype=np.uint64)
    pairs[0, 0] = 0
    np.cumsum(lens[:-1], out=pairs[1:, 0])
    pairs[:, 0] += np.uint64(buf.ctypes.data)
    pairs[:, 1] = lens
    return pairs.ctypes.data_as(POINTER(Bytes)), (buf, pairs, blob)


def int32_array(values):
    """A contiguous int32 array and its pointer (values must fit in i32)."""
    import numpy as np

    a = np.ascontiguousarray(values, dtype=np.int32)
    if a.size == 0:
        a = np.zeros(1, np.int32)
    return a.ctypes.data_as(POINTER(c_int32)), a
