"""vLLM v1 KV connector over the B200 engine server.

Configure vLLM with ``kv_connector="PegaKVConnector"`` and
``kv_connector_module_path="pegaflow_b200.connector"``; the server is
``python -m pegaflow_b200.server`` (endpoint from PEGAFLOW_ENGINE_ENDPOINT).
PEGAFLOW_LAYERWISE=1 restores cached KV inside the forward, one layer at a
time, so attention on layer l starts once layer l is in HBM.
"""

from __future__ import annotations

from typing import Any, Iterable, Optional

from .scheduler import SchedulerSide
from .state import (  # noqa: F401
    ENGINE_ENDPOINT,
    LAYERWISE,
    ConnectorContext,
    LoadIntent,
    PegaConnectorMetadata,
    RequestTracker,
    SaveIntent,
    derive_namespace,
    log,
    namespace_from_factors,
    resolve_instance_id,
)
from .worker import WorkerSide

try:
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_V1, KVConnectorRole
except Exception:  # vLLM absent: the sides above still work on their own
    KVConnectorBase_V1, KVConnectorRole = object, None


class PegaKVConnector(KVConnectorBase_V1):
    """KVConnectorBase_V1 facade dispatching to the scheduler or worker side
    (the reference facade: python/pegaflow/connector/__init__.py:33-212)."""

    def __init__(self, vllm_config, role, kv_cache_config=None):
        try:
            super().__init__(vllm_config, role, kv_cache_config)
        except TypeError:
            super().__init__(vllm_config, role)
        import torch

        from ..client import EngineRpcClient

        tp_size = vllm_config.parallel_config.tensor_parallel_size
        tp_rank = device_id = None
        if role == KVConnectorRole.WORKER:
            from vllm.distributed.parallel_state import get_tensor_model_parallel_rank

            tp_rank = get_tensor_model_parallel_rank()
            if torch.cuda.is_available():
                device_id = torch.cuda.current_device()
        self._ctx = ConnectorContext(
            instance_id=resolve_instance_id(vllm_config),
            namespace=derive_namespace(vllm_config, tp_size),
            block_size=vllm_config.cache_config.block_size,
            num_layers=getattr(vllm_config.model_config.hf_text_config, "num_hidden_layers", 0),
            tp_size=tp_size,
            tp_rank=tp_rank,
            device_id=device_id,
            engine_client=EngineRpcClient(ENGINE_ENDPOINT),
            layerwise=LAYERWISE,
        )
        self._scheduler: Optional[SchedulerSide] = None
        self._worker: Optional[WorkerSide] = None
        if role == KVConnectorRole.SCHEDULER:
            self._scheduler = SchedulerSide(self._ctx)
        else:
            self._worker = WorkerSide(self._ctx)

    # -- worker side ------------------------------------------------------------
    def register_kv_caches(self, kv_caches: dict) -> None:
        if self._worker:
            self._worker.register_kv_caches(kv_caches)

    def start_load_kv(self, forward_context, **kwargs: Any) -> None:
        meta = self._get_connector_metadata() if self._worker else None
        if meta is not None:
            self._worker.start_load_kv(meta, forward_context)

    def wait_for_layer_load(self, layer_name: str) -> None:
        if self._worker:
            self._worker.wait_for_layer_load(layer_name)

    def save_kv_layer(self, layer_name: str, kv_layer, attn_metadata, **kwargs: Any) -> None:
        meta = self._get_connector_metadata() if self._worker else None
        if meta is not None:
            self._worker.save_kv_layer(meta, layer_name, kv_layer, attn_metadata)

    def wait_for_save(self) -> None:
        if self._worker:
            self._worker.wait_for_save()

    def get_finished(self, finished_req_ids: set) -> tuple:
        return self._worker.get_finished(finished_req_ids) if self._worker else (None, None)

    def unregister_context(self) -> None:
        if self._worker:
            self._worker.unregister_context()

    # -- scheduler side -----------------------------------------------------------
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        if not self._scheduler:
            return 0, False
        return self._scheduler.get_num_new_matched_tokens(request, num_computed_tokens)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        if self._scheduler:
            self._scheduler.update_state_after_alloc(request, blocks, num_external_tokens)

    def build_connector_meta(self, scheduler_output) -> PegaConnectorMetadata:
        return self._scheduler.build_connector_meta(scheduler_output) if self._scheduler else PegaConnectorMetadata()

    def update_connector_output(self, connector_output) -> None:
        if self._scheduler:
            self._scheduler.update_connector_output(connector_output)

    def request_finished(self, request, block_ids):
        return self._scheduler.request_finished(request, block_ids) if self._scheduler else (False, None)

    def take_events(self) -> Iterable:
        return ()

    def get_block_ids_with_load_errors(self) -> set:
        return set()

    def shutdown(self) -> None:
        if self._worker:
            self._worker.shutdown()


__all__ = ["PegaKVConnector", "PegaConnectorMetadata", "SchedulerSide", "WorkerSide", "ConnectorContext"]
