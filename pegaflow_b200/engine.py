"""In-process engine and load-state classes with the reference's Python surface.

``PegaEngine`` and ``PyLoadState`` keep the names, argument order and error
behaviour (``RuntimeError`` carrying the engine's message) of the PyO3 classes
in python/src/lib.rs:89-261 and :539-574. ``PegaEngine`` adds the save calls
of the core engine (pegaflow-core/src/lib.rs:497-550), which the reference only
reaches through its gRPC server.
"""

from __future__ import annotations

import ctypes
from ctypes import byref, c_char_p, c_uint8, c_uint64, c_void_p
from typing import Iterable, Optional, Sequence

from . import _native as N
from .transfer import Executor

DEFAULT_POOL_BYTES = 30 * 1024 * 1024 * 1024  # pegaflow-core/src/lib.rs:56


class PegaEngine:
    """PegaEngine (python/src/lib.rs:89-261) backed by the B200 C++ engine.

    With no arguments it allocates the reference's default 30 GiB pinned pool.
    ``pool_kind="host"`` builds the engine over plain pageable memory for
    host-logic tests: registration, queries and bookkeeping work, transfers
    raise.
    """

    def __init__(
        self,
        pool_size: int = DEFAULT_POOL_BYTES,
        use_hugepages: bool = False,
        *,
        write_combined: bool = True,
        enable_lfu_admission: bool = True,
        hint_value_size_bytes: int = 0,
        pre_evict: Optional[tuple[int, int, int]] = None,
        pool_kind: str = "pinned",
        executor: Optional[dict] = None,
        dfs_root: Optional[str] = None,
        dfs_quota: int = 0,
        dfs_scan_interval_ms: int = 0,
        dfs_max_pack_size: int = 0,
        numa_pools: str = "off",
    ):
        """``dfs_root`` turns on the packed-file tier: sealed blocks are
        written through to ``{dfs_root}/{namespace}/{uuid}.bin`` and read
        back when ``query_prefetch`` finds them missing from the pool.

        ``numa_pools`` splits the pool for an engine that drives several
        GPUs: "off" (one pool, the default), "node" (one pool per NUMA node of
        the visible GPUs) or "device" (one pool per GPU). Each pool sits on
        its GPUs' NUMA node, and a save allocates from its GPU's pool."""
        modes = {"off": 0, "node": 1, "device": 2}
        if numa_pools not in modes:
            raise ValueError(f"numa_pools must be one of {sorted(modes)}, not {numa_pools!r}")
        cfg = N.EngineConfig()
        N.lib.pf_engine_config_default(byref(cfg))
        cfg.numa_pools = modes[numa_pools]
        cfg.pool_bytes = pool_size
        cfg.use_hugepages = 1 if use_hugepages else 0
        cfg.write_combined = 1 if write_combined else 0
        cfg.enable_lfu_admission = 1 if enable_lfu_admission else 0
        cfg.hint_value_size_bytes = hint_value_size_bytes
        cfg.pool_kind = N.PF_POOL_HOST if pool_kind == "host" else N.PF_POOL_PINNED
        if pre_evict is not None:
            cfg.pre_evict_enabled = 1
            cfg.pre_evict_threshold_bytes, cfg.pre_evict_target_bytes, cfg.pre_evict_interval_ms = pre_evict
        if executor:
            modes = {"auto": N.PF_MODE_AUTO, "staged": N.PF_MODE_STAGED, "direct": N.PF_MODE_DIRECT}
            kernels = {"auto": N.PF_COPY_KERNEL_AUTO, "registers": N.PF_COPY_KERNEL_REGISTERS,
                       "bulk": N.PF_COPY_KERNEL_BULK}
            for k, v in executor.items():
                if k.endswith("_mode"):
                    v = modes[v]
                elif k == "copy_kernel" and isinstance(v, str):
                    v = kernels[v]
                setattr(cfg.executor, k, v)
        root = dfs_root.encode() if dfs_root else None  # kept alive across the create call
        cfg.dfs_root = root
        cfg.dfs_quota_bytes = dfs_quota
        cfg.dfs_scan_interval_ms = dfs_scan_interval_ms
        cfg.dfs_max_pack_size = dfs_max_pack_size
        h = c_void_p()
        N.check(N.lib.pf_engine_create(byref(cfg), byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            N.lib.pf_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- reference PyO3 surface ------------------------------------------------

    def register_context_layer(
        self,
        instance_id: str,
        namespace: str,
        device_id: int,
        layer_name: str,
        data_ptr: int,
        size_bytes: int,
        num_blocks: int,
        bytes_per_block: int,
        kv_stride_bytes: int,
        segments: int,
        tp_rank: int,
        tp_size: int,
        num_layers: int,
    ) -> None:
        N.check(
            N.lib.pf_engine_register_context_layer(
                self._h,
                instance_id.encode(),
                namespace.encode(),
                device_id,
                layer_name.encode(),
                data_ptr,
                size_bytes,
                num_blocks,
                bytes_per_block,
                kv_stride_bytes,
                segments,
                tp_rank,
                tp_size,
                num_layers,
            )
        )

    def unregister_instance(self, instance_id: str) -> None:
        N.check(N.lib.pf_engine_unregister_instance(self._h, instance_id.encode()))

    def count_prefix_hit_blocks(self, instance_id: str, block_hashes: Sequence[bytes]) -> int:
        arr, keep = N.bytes_array(block_hashes)
        out = c_uint64()
        N.check(N.lib.pf_engine_count_prefix_hit_blocks(self._h, instance_id.encode(), arr, len(block_hashes), byref(out)))
        del keep
        return out.value

    def query_prefetch(self, instance_id: str, block_hashes: Sequence[bytes]) -> dict:
        """count_prefix_hit_blocks_async (pegaflow-core/src/lib.rs:855-942):
        ``prefetch_state`` is "ready", "loading" (blocks are being read back
        from the packed-file tier: ask again) or "partial_miss"."""
        arr, keep = N.bytes_array(block_hashes)
        s = N.PrefetchStatus()
        N.check(N.lib.pf_engine_query_prefetch(self._h, instance_id.encode(), arr, len(block_hashes), byref(s)))
        del keep
        return {"hit_blocks": s.hit_blocks, "prefetch_state": ("ready", "loading", "partial_miss")[s.state],
                "loading_blocks": s.loading_blocks, "missing_blocks": s.missing_blocks}

    def dfs_stats(self) -> dict:
        s = N.DfsStats()
        N.check(N.lib.pf_engine_dfs_stats(self._h, byref(s)))
        return {f: getattr(s, f) for f, _ in N.DfsStats._fields_}

    def dfs_flush(self, timeout_s: float = 30.0) -> bool:
        """Wait for queued packed-file writes and reads; False on timeout."""
        idle = ctypes.c_int()
        N.check(N.lib.pf_engine_dfs_flush(self._h, timeout_s, byref(idle)))
        return bool(idle.value)

    def dfs_check_quota(self) -> None:
        N.check(N.lib.pf_engine_dfs_check_quota(self._h))

    def batch_load_kv_blocks(
        self,
        instance_id: str,
        tp_rank: int,
        device_id: int,
        load_state_shm: str,
        layer_names: Sequence[str],
        block_ids: Sequence[int],
        block_hashes: Sequence[bytes],
    ) -> None:
        names = (c_char_p * max(1, len(layer_names)))(*[n.encode() for n in layer_names])
        # The reference pairs ids with hashes up to the shorter list
        # (lib.rs:1032-1033); the C call takes one count for both arrays.
        n = min(len(block_ids), len(block_hashes))
        block_ids, block_hashes = list(block_ids)[:n], list(block_hashes)[:n]
        ids, ids_keep = N.int32_array(block_ids)
        arr, keep = N.bytes_array(block_hashes)
        N.check(
            N.lib.pf_engine_batch_load_kv_blocks(
                self._h,
                instance_id.encode(),
                tp_rank,
                device_id,
                load_state_shm.encode(),
                names,
                len(layer_names),
                ids,
                arr,
                len(block_hashes),
            )
        )
        del keep, ids_keep

    def save_request(self, request: bytes) -> None:
        """The server's Save RPC on a request's wire bytes (engine.proto
        SaveRequest), decoded by the library: batch_save_kv_blocks without
        per-layer Python lists."""
        N.check(N.lib.pf_engine_save_request(self._h, request, len(request)))

    def load_request(self, request: bytes) -> None:
        """The server's Load RPC on a request's wire bytes (engine.proto
        LoadRequest), decoded by the library."""
        N.check(N.lib.pf_engine_load_request(self._h, request, len(request)))

    # -- core engine calls the reference exposes through its server ------------

    def batch_save_kv_blocks(
        self,
        instance_id: str,
        tp_rank: int,
        device_id: int,
        saves: Iterable[tuple[str, Sequence[int], Sequence[bytes]]],
    ) -> None:
        """PegaEngine::batch_save_kv_blocks_from_ipc (pegaflow-core/src/lib.rs:497-520)."""
        saves = list(saves)
        entries = (N.SaveEntry * max(1, len(saves)))()
        keep = []
        converted = {}  # the same hash list object is often shared by every layer
        converted_ids = {}  # and so is the block id list
        for i, (layer, ids, hashes) in enumerate(saves):
            name = layer.encode()
            if id(ids) not in converted_ids:
                converted_ids[id(ids)] = (ids, *N.int32_array(ids))
            _, id_ptr, id_keep = converted_ids[id(ids)]
            if id(hashes) not in converted:
                converted[id(hashes)] = (hashes, *N.bytes_array(hashes))
            _, h_ptr, hk = converted[id(hashes)]
            keep += [name, id_keep, hk]
            entries[i].layer_name = name
            entries[i].block_ids = id_ptr
            entries[i].n_ids = len(ids)
            entries[i].block_hashes = h_ptr
            entries[i].n_hashes = len(hashes)
        N.check(N.lib.pf_engine_batch_save_kv_blocks(self._h, instance_id.encode(), tp_rank, device_id, entries, len(saves)))
        del keep

    def save_kv_blocks(
        self,
        instance_id: str,
        tp_rank: int,
        device_id: int,
        layer_name: str,
        block_ids: Sequence[int],
        block_hashes: Sequence[bytes],
    ) -> None:
        """PegaEngine::save_kv_blocks_from_ipc (pegaflow-core/src/lib.rs:528-550)."""
        self.batch_save_kv_blocks(instance_id, tp_rank, device_id, [(layer_name, block_ids, block_hashes)])

    # -- extras -----------------------------------------------------------------

    def wait_loads(self, device_id: int, timeout_s: float = 60.0) -> None:
        N.check(N.lib.pf_engine_wait_loads(self._h, device_id, timeout_s))

    def pool_usage(self) -> tuple[int, int, int]:
        used, total, largest = c_uint64(), c_uint64(), c_uint64()
        N.check(N.lib.pf_engine_pool_usage(self._h, byref(used), byref(total), byref(largest)))
        return used.value, total.value, largest.value

    def slot_info(self, namespace: str, block_hash: bytes, slot: int) -> tuple[int, int, int]:
        """(k_ptr, v_ptr, size) of a sealed block's slot; v_ptr 0 when contiguous."""
        buf = (c_uint8 * max(1, len(block_hash))).from_buffer_copy(block_hash or b"\0")
        k, v, s = c_uint64(), c_uint64(), c_uint64()
        N.check(
            N.lib.pf_engine_slot_info(
                self._h, namespace.encode(), buf, len(block_hash), slot, byref(k), byref(v), byref(s)
            )
        )
        return k.value, v.value, s.value

    def metrics(self) -> dict:
        m = N.EngineMetrics()
        N.check(N.lib.pf_engine_metrics_get(self._h, byref(m)))
        return {f: getattr(m, f) for f, _ in N.EngineMetrics._fields_}

    def executor(self, device_id: int) -> Executor:
        h = c_void_p()
        N.check(N.lib.pf_engine_executor(self._h, device_id, byref(h)))
        return Executor(device_id, _handle=h.value)


class PyLoadState:
    """Batch-level load completion flag in shared memory (python/src/lib.rs:539-574).

    State values: 0 pending, 1 success, <0 error. The creating object owns the
    shared-memory object and unlinks it when closed or collected.
    """

    def __init__(self, n_layers: int = 0):
        """n_layers > 0 adds one completion word per layer of the load request
        (an extension after the version-1 bytes, which stay readable by the
        reference's LoadState::attach)."""
        h = c_void_p()
        if n_layers:
            N.check(N.lib.pf_load_state_create_layers(n_layers, byref(h)))
        else:
            N.check(N.lib.pf_load_state_create(byref(h)))
        self._h = h

    @classmethod
    def attach(cls, shm_name: str) -> "PyLoadState":
        """LoadState::attach (pegaflow-core/src/sync_state.rs:145-155); does not own the object."""
        self = cls.__new__(cls)
        h = c_void_p()
        N.check(N.lib.pf_load_state_attach(shm_name.encode(), byref(h)))
        self._h = h
        return self

    def shm_name(self) -> str:
        return N.lib.pf_load_state_name(self._h).decode()

    def get_state(self) -> int:
        return int(N.lib.pf_load_state_get(self._h))

    def is_ready(self) -> bool:
        return self.get_state() != 0

    def layer_count(self) -> int:
        return int(N.lib.pf_load_state_layer_count(self._h))

    def layer_ready(self, layer: int) -> bool:
        """True once the bytes of layer `layer` (index into the load's
        layer_names) are in place."""
        return int(N.lib.pf_load_state_layer_get(self._h, layer)) == 1

    def wait_layer(self, layer: int, timeout_s: float = 5.0) -> bool:
        """Poll until layer `layer` is in place (True), the load failed or the
        timeout ran out (False)."""
        import time

        deadline = time.monotonic() + timeout_s
        while True:
            if self.layer_ready(layer):
                return True
            if self.get_state() < 0 or time.monotonic() > deadline:
                return False
            time.sleep(0)

    def set_completed(self) -> None:
        N.lib.pf_load_state_set_completed(self._h)

    def set_error(self) -> None:
        N.lib.pf_load_state_set_error(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            N.lib.pf_load_state_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def request_instance_id(request: bytes) -> str:
    """Field 1 (instance_id) of a Save or Load request's wire bytes."""
    cap = 4096
    out = ctypes.create_string_buffer(cap)
    n = c_uint64()
    N.check(N.lib.pf_request_instance_id(request, len(request), out, cap, byref(n)))
    return out.raw[: n.value].decode("utf-8", "replace")
