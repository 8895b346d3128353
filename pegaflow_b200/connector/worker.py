"""Worker side of the vLLM connector: registers KV tensors with the engine
server, batches per-layer saves on a background thread, issues loads with a
LoadState, reports completion, and (layer-wise mode) waits per layer.

RPC composition follows the reference worker (python/pegaflow/connector/
worker.py:80-427; pinned by tests/golden/save_batches.json and
load_requests.json). Two changes: a save waits only for the CUDA event
recorded when vLLM handed the layer over, not for the whole device
(worker.py:395 calls torch.cuda.synchronize()); and wait_for_layer_load waits
for that layer's completion word instead of returning at once
(worker.py:288-289).
"""

from __future__ import annotations

import pickle
import queue
import threading
import time
from dataclasses import dataclass
from typing import Any, Optional

from .state import ConnectorContext, PegaConnectorMetadata, log

LAYER_WAIT_S = 30.0


@dataclass
class _SaveTask:
    layer_name: str
    attn_metadata: Any
    metadata: PegaConnectorMetadata
    request_ids: list
    ready: Any = None  # CUDA event recorded after the layer's KV was written


def _layout(kv_cache):
    """(num_blocks, bytes_per_block, kv_stride_bytes, segments) as the worker
    derives them from the tensor (worker.py:100-115)."""
    shape, stride, elt = tuple(kv_cache.shape), tuple(kv_cache.stride()), kv_cache.element_size()
    if len(shape) >= 2 and shape[0] == 2:
        return shape[1], stride[1] * elt, stride[0] * elt, 2
    return shape[0], stride[0] * elt, 0, 1


class WorkerSide:
    def __init__(self, ctx: ConnectorContext, load_state_factory=None, wrapper_factory=None):
        self._ctx = ctx
        self._new_load_state = load_state_factory
        self._wrap = wrapper_factory
        self._save_q: "queue.Queue[Optional[_SaveTask]]" = queue.Queue()
        self._save_lock = threading.Lock()
        self._pending_layers: dict[str, int] = {}
        self._completed_saves: set = set()
        self._finished: set = set()
        self._current_save_intents: set = set()
        self._load_lock = threading.Lock()
        self._loads: dict[str, tuple] = {}  # shm name -> (LoadState, request ids)
        self._layer_index: dict[str, int] = {}
        self._layer_state = None
        self._layers: list[str] = []
        self._save_thread = threading.Thread(target=self._save_loop, daemon=True, name="PegaSaveWorker")
        self._save_thread.start()

    # ------------------------------------------------------------------ lifecycle

    def shutdown(self) -> None:
        # Saves already queued go out before the instance is unregistered (the
        # reference unregisters first, worker.py:60-63, and those saves fail).
        self._save_q.put(None)
        self._save_thread.join()
        self.unregister_context()

    def unregister_context(self) -> None:
        if not self._layers:
            return
        if self._ctx.tp_rank == 0:  # one rank unregisters the shared instance (worker.py:69-76)
            ok, msg = self._ctx.engine_client.unregister_context(self._ctx.instance_id)
            if not ok:
                log.warning("unregister_context failed: %s", msg)
        self._layers = []

    def register_kv_caches(self, kv_caches: dict) -> None:
        if self._ctx.device_id is None:
            raise RuntimeError("CUDA device id is unknown; cannot register KV caches")
        if self._wrap is None:
            from ..ipc import CudaIPCWrapper

            self._wrap = CudaIPCWrapper
        self._layers = list(kv_caches)
        for name, kv in kv_caches.items():
            if kv.storage_offset() != 0:
                raise RuntimeError(f"KV cache for {name} must start at its storage's first byte")
            num_blocks, bytes_per_block, kv_stride, segments = _layout(kv)
            if bytes_per_block == 0:
                raise RuntimeError(f"Invalid bytes_per_block for {name}: stride={tuple(kv.stride())}")
            ok, msg = self._ctx.engine_client.register_context(
                self._ctx.instance_id, self._ctx.namespace, self._ctx.tp_rank, self._ctx.tp_size,
                self._ctx.device_id, self._ctx.num_layers, name, pickle.dumps(self._wrap(kv)), num_blocks,
                bytes_per_block, kv_stride, segments)
            if not ok:
                raise RuntimeError(f"Register context failed for {name}: {msg}")
        log.info("registered %d KV cache layers for instance %s", len(kv_caches), self._ctx.instance_id)

    # ------------------------------------------------------------------ loads

    def start_load_kv(self, metadata: PegaConnectorMetadata, forward_context) -> None:
        self._current_save_intents = set(metadata.save_intents)
        if not metadata.load_intents:
            return
        ids, hashes, req_ids = [], [], []
        for req_id, intent in metadata.load_intents.items():
            ids.extend(intent.block_ids)
            hashes.extend(intent.block_hashes)
            req_ids.append(req_id)
        if not ids:
            return
        layers = [n for n, layer in forward_context.no_compile_layers.items() if hasattr(layer, "kv_cache")]
        if not layers:
            return
        if self._new_load_state is None:
            from ..engine import PyLoadState

            self._new_load_state = PyLoadState
        state = self._new_load_state(len(layers))
        ok, msg = self._ctx.engine_client.load(self._ctx.instance_id, self._ctx.tp_rank, self._ctx.device_id,
                                               state.shm_name(), layers, ids, hashes)
        if not ok:
            raise RuntimeError(f"Load request failed: {msg}")
        with self._load_lock:
            self._loads[state.shm_name()] = (state, set(req_ids))
            self._layer_index = {n: i for i, n in enumerate(layers)}
            self._layer_state = state

    def wait_for_layer_load(self, layer_name: str) -> None:
        """Block until this layer's restored KV is in place (layer-wise mode)."""
        state, idx = self._layer_state, self._layer_index.get(layer_name)
        if not self._ctx.layerwise or state is None or idx is None:
            return
        if not state.wait_layer(idx, LAYER_WAIT_S):
            log.error("layer %s of load %s not restored (state %d)", layer_name, state.shm_name(),
                      state.get_state())

    # ------------------------------------------------------------------ saves

    def save_kv_layer(self, metadata: PegaConnectorMetadata, layer_name: str, kv_layer, attn_metadata) -> None:
        request_ids = list(metadata.save_intents)
        if not request_ids:
            return
        with self._save_lock:
            for r in request_ids:
                self._pending_layers.setdefault(r, len(self._layers))
        ready = None
        try:
            import torch

            if torch.cuda.is_available():
                ready = torch.cuda.Event()
                ready.record()
        except Exception:
            ready = None
        self._save_q.put(_SaveTask(layer_name, attn_metadata, metadata, request_ids, ready))

    def wait_for_save(self) -> None:
        with self._save_lock:
            skipped = self._current_save_intents - set(self._pending_layers)
            if skipped:
                # save_kv_layer never ran for them (e.g. a captured CUDA graph step)
                self._completed_saves |= skipped
            self._current_save_intents = set()

    def _save_loop(self) -> None:
        while True:
            task = self._save_q.get()
            if task is None:
                return
            batch = [task]
            stop = False
            while True:
                try:
                    t = self._save_q.get_nowait()
                except queue.Empty:
                    break
                if t is None:
                    stop = True
                    break
                batch.append(t)
            self.process_save_batch(batch)
            if stop:
                return

    def process_save_batch(self, batch: list) -> None:
        """One save RPC for a batch of per-layer tasks (worker.py:372-427)."""
        by_layer: dict[str, tuple[list, list]] = {}
        request_ids: list = []
        for task in batch:
            request_ids.extend(task.request_ids)
            if getattr(task.attn_metadata, "block_table", None) is None:
                continue
            for intent in task.metadata.save_intents.values():
                if not intent.block_ids:
                    continue
                ids, hs = by_layer.setdefault(task.layer_name, ([], []))
                ids.extend(intent.block_ids)
                hs.extend(intent.block_hashes)
        if by_layer:
            for task in batch:
                if task.ready is not None:
                    task.ready.synchronize()  # the layer's KV is written before the server reads it
            saves = [(name, ids, hs) for name, (ids, hs) in by_layer.items()]
            try:
                ok, msg = self._ctx.engine_client.save(self._ctx.instance_id, self._ctx.tp_rank,
                                                       self._ctx.device_id, saves)
                if not ok:
                    log.error("save batch failed: %s (continuing without save)", msg)
            except Exception as e:  # the request still completes without its save (worker.py:417-424)
                log.error("save RPC failed: %s (continuing without save)", e)
        self._release(request_ids)

    def _release(self, request_ids: list) -> None:
        with self._save_lock:
            for r in request_ids:
                if r in self._pending_layers:
                    self._pending_layers[r] -= 1
                    if self._pending_layers[r] <= 0:
                        del self._pending_layers[r]
                        self._completed_saves.add(r)

    # ------------------------------------------------------------------ completion

    def get_finished(self, finished_req_ids: set) -> tuple:
        sending = recving = None
        with self._save_lock:
            self._finished |= finished_req_ids & set(self._pending_layers)
            done = (self._completed_saves & self._finished) | (self._completed_saves & finished_req_ids)
            if done:
                self._completed_saves -= done
                self._finished -= done
                sending = done
        with self._load_lock:
            done_loads = [shm for shm, (s, _) in self._loads.items() if s.is_ready()]
            reqs = set()
            for shm in done_loads:
                state, ids = self._loads.pop(shm)
                if state.get_state() < 0:
                    log.error("async load failed (state %d) for %s", state.get_state(), ids)
                reqs |= ids
                if self._layer_state is state:
                    self._layer_state, self._layer_index = None, {}
            # In layer-wise mode vLLM does not wait for these requests.
            if reqs and not self._ctx.layerwise:
                recving = reqs
        return sending, recving
