"""Request bookkeeping shared by the scheduler and worker sides of the vLLM
connector: load/save intents, the per-request tracker and the context.

The behaviour follows the reference connector (python/pegaflow/connector/
common.py:44-302): a lookup opens a load window over the cache hits not yet
computed by vLLM's own prefix cache; block allocation fills it; the first
scheduling consumes it as a LoadIntent; SaveIntents cover newly completed
blocks as tokens get scheduled.
"""

from __future__ import annotations

import enum
import hashlib
import logging
import os
import uuid
from dataclasses import dataclass, field
from typing import Any, Optional

log = logging.getLogger("pegaflow_b200.connector")

ENGINE_ENDPOINT = os.environ.get("PEGAFLOW_ENGINE_ENDPOINT", "http://127.0.0.1:50055")
# Layer-wise restore: load synchronously inside the forward and wait per layer
# (vLLM calls wait_for_layer_load before each attention layer).
LAYERWISE = os.environ.get("PEGAFLOW_LAYERWISE", "0") not in ("", "0", "false", "False")


@dataclass(frozen=True)
class ConnectorContext:
    instance_id: str
    namespace: str
    block_size: int
    num_layers: int
    tp_size: int
    tp_rank: Optional[int]
    device_id: Optional[int]
    engine_client: Any
    layerwise: bool = False


class RequestPhase(enum.Enum):
    LOOKUP = "lookup"
    LOADING = "loading"
    ACTIVE = "active"
    DRAINING = "draining"
    DONE = "done"


@dataclass(frozen=True)
class LoadIntent:
    block_ids: tuple
    block_hashes: tuple
    num_tokens: int


@dataclass(frozen=True)
class SaveIntent:
    block_ids: tuple
    block_hashes: tuple


@dataclass
class _LoadWindow:
    hit_blocks: int
    computed_blocks: int
    allocated: list = field(default_factory=list)
    external_tokens: int = 0

    def intent(self, hashes: tuple, block_size: int) -> Optional[LoadIntent]:
        if self.external_tokens <= 0 or self.hit_blocks <= self.computed_blocks:
            return None
        end = min(self.hit_blocks, len(self.allocated), len(hashes))
        if end <= self.computed_blocks:
            return None
        lo = self.computed_blocks
        return LoadIntent(tuple(self.allocated[lo:end]), tuple(hashes[lo:end]), (end - lo) * block_size)


class RequestTracker:
    """KV cache state of one request across scheduling steps."""

    def __init__(self, request_id: str, block_hashes, block_size: int, num_layers: int):
        self.request_id = request_id
        self.hashes = tuple(block_hashes)
        self.block_size = block_size
        self.total_layers = num_layers
        self.saved_layers = 0
        self.finished = False
        self._window: Optional[_LoadWindow] = None
        self._allocated: list = []
        self._scheduled_tokens = 0
        self._stored_blocks = 0

    @property
    def phase(self) -> RequestPhase:
        if self._window is not None:
            return RequestPhase.LOADING
        if not self.finished:
            return RequestPhase.ACTIVE
        return RequestPhase.DRAINING if self.saved_layers < self.total_layers else RequestPhase.DONE

    def on_lookup(self, hit_blocks: int, computed_blocks: int) -> None:
        # A new lookup (also after a preemption) starts a fresh window.
        self._window = _LoadWindow(hit_blocks, computed_blocks) if hit_blocks > computed_blocks else None
        self._allocated = []

    def on_alloc(self, block_ids, num_external_tokens: int) -> None:
        self._allocated.extend(block_ids)
        if self._window is not None:
            self._window.allocated.extend(block_ids)
            if num_external_tokens > 0:
                self._window.external_tokens = num_external_tokens

    def consume_load_intent(self) -> Optional[LoadIntent]:
        w, self._window = self._window, None
        return None if w is None else w.intent(self.hashes, self.block_size)

    def on_scheduled(self, num_tokens: int) -> None:
        self._scheduled_tokens += num_tokens

    def consume_save_intent(self) -> Optional[SaveIntent]:
        ready = min(len(self.hashes), len(self._allocated), self._scheduled_tokens // self.block_size)
        if ready <= self._stored_blocks:
            return None
        lo, self._stored_blocks = self._stored_blocks, ready
        return SaveIntent(tuple(self._allocated[lo:ready]), tuple(self.hashes[lo:ready]))

    def on_layer_saved(self) -> None:
        self.saved_layers += 1

    def on_finished(self) -> None:
        self.finished = True

    def should_hold_blocks(self) -> bool:
        return self.finished and self._stored_blocks > 0 and self.saved_layers < self.total_layers

    def is_done(self) -> bool:
        return self.phase == RequestPhase.DONE


def _metadata_base():
    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorMetadata

        return KVConnectorMetadata
    except Exception:  # vLLM absent: a plain base keeps the class usable in tests
        return object


class PegaConnectorMetadata(_metadata_base()):
    """Scheduler -> worker message of one step: request id -> intents."""

    def __init__(self, load_intents=None, save_intents=None):
        super().__init__()
        self.load_intents: dict = load_intents or {}
        self.save_intents: dict = save_intents or {}

    def __repr__(self) -> str:
        return f"PegaConnectorMetadata(loads={len(self.load_intents)}, saves={len(self.save_intents)})"


def resolve_instance_id(vllm_config, dp_rank_suffix: bool = True) -> str:
    """kv_transfer_config.engine_id, else vLLM's instance id or
    PEGAFLOW_INSTANCE_ID, else a random id; '_dp{rank}' appended under data
    parallelism (the reference's rules, common.py:254-280)."""
    instance_id = vllm_config.kv_transfer_config.engine_id
    if instance_id:
        return instance_id
    instance_id = vllm_config.instance_id or os.environ.get("PEGAFLOW_INSTANCE_ID", "") or uuid.uuid4().hex
    pc = vllm_config.parallel_config
    if dp_rank_suffix and pc.data_parallel_size > 1 and pc.data_parallel_rank_local is not None:
        instance_id = f"{instance_id}_dp{pc.data_parallel_rank_local}"
    return instance_id


def namespace_from_factors(factors: dict) -> str:
    """First 8 hex digits of sha256(str(sorted(factors.items()))) — the same
    derivation as the reference (common.py:283-302), so workers of either
    implementation that serve the same model share cached blocks."""
    return hashlib.sha256(str(sorted(factors.items())).encode()).hexdigest()[:8]


def derive_namespace(vllm_config, tp_size: int) -> str:
    mc, cc = vllm_config.model_config, vllm_config.cache_config
    return namespace_from_factors({
        "model": mc.model,
        "dtype": str(mc.dtype),
        "tp_size": tp_size,
        "num_kv_heads": mc.get_total_num_kv_heads(),
        "head_size": mc.get_head_size(),
        "num_hidden_layers": mc.get_total_num_hidden_layers(),
        "cache_dtype": str(cc.cache_dtype),
    })
