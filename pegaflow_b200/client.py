"""EngineRpcClient: the reference's blocking gRPC client (python/src/lib.rs:263-528)
over grpcio, with the same methods, arguments and return shapes: (ok, message)
tuples, and a dict for ``query``. Transport and RPC failures raise
RuntimeError, as the PyO3 client does."""

from __future__ import annotations

from typing import Optional, Sequence

import grpc

from . import proto as P

DEFAULT_ENDPOINT = "http://127.0.0.1:50055"  # python/src/lib.rs:268

_PREFETCH = {P.PREFETCH_READY: "ready", P.PREFETCH_LOADING: "loading", P.PREFETCH_PARTIAL_MISS: "partial_miss"}


def _target(endpoint: str) -> str:
    for scheme in ("http://", "https://", "grpc://"):
        if endpoint.startswith(scheme):
            return endpoint[len(scheme):].rstrip("/")
    return endpoint


class EngineRpcClient:
    def __init__(self, endpoint: Optional[str] = None, connect_timeout_s: float = 0.5):
        """Connects eagerly with a 500 ms timeout and keeps the channel, as the
        reference client does (python/src/lib.rs:265-290)."""
        self._endpoint = endpoint or DEFAULT_ENDPOINT
        self._channel = grpc.insecure_channel(
            _target(self._endpoint),
            options=[("grpc.keepalive_time_ms", 30000), ("grpc.keepalive_permit_without_calls", 1),
                     ("grpc.max_receive_message_length", 256 << 20),
                     ("grpc.max_send_message_length", 256 << 20)])
        try:
            grpc.channel_ready_future(self._channel).result(timeout=connect_timeout_s)
        except grpc.FutureTimeoutError:
            self._channel.close()
            raise RuntimeError(f"failed to connect to engine server at {self._endpoint}: timed out") from None
        self._stubs = {
            rpc: self._channel.unary_unary(f"/{P.SERVICE}/{rpc}", request_serializer=P.M[req].SerializeToString,
                                           response_deserializer=P.M[resp].FromString)
            for rpc, (req, resp) in P.METHODS.items()
        }

    def _call(self, rpc: str, request):
        try:
            return self._stubs[rpc](request)
        except grpc.RpcError as e:
            raise RuntimeError(f"rpc RPC failed: status: {e.code().name}, message: {e.details()!r}") from None

    @staticmethod
    def _status(method: str, resp) -> tuple[bool, str]:
        if not resp.HasField("status"):
            raise RuntimeError(f"{method} response missing status")
        return resp.status.ok, resp.status.message

    def endpoint(self) -> str:
        return self._endpoint

    def health(self) -> tuple[bool, str]:
        return self._status("health", self._call("Health", P.HealthRequest()))

    def register_context(self, instance_id: str, namespace: str, tp_rank: int, tp_size: int, device_id: int,
                         num_layers: int, layer_name: str, wrapper_bytes: bytes, num_blocks: int,
                         bytes_per_block: int, kv_stride_bytes: int, segments: int) -> tuple[bool, str]:
        req = P.RegisterContextRequest(
            instance_id=instance_id, tp_rank=tp_rank, tp_size=tp_size, device_id=device_id, num_layers=num_layers,
            layer_name=layer_name, wrapper_bytes=wrapper_bytes, num_blocks=num_blocks,
            bytes_per_block=bytes_per_block, kv_stride_bytes=kv_stride_bytes, segments=segments, namespace=namespace)
        return self._status("register_context", self._call("RegisterContext", req))

    def save(self, instance_id: str, tp_rank: int, device_id: int,
             saves: Sequence[tuple[str, Sequence[int], Sequence[bytes]]]) -> tuple[bool, str]:
        req = P.SaveRequest(instance_id=instance_id, tp_rank=tp_rank, device_id=device_id,
                            saves=[P.SaveLayer(layer_name=n, block_ids=list(ids), block_hashes=list(hs))
                                   for n, ids, hs in saves])
        return self._status("save", self._call("Save", req))

    def load(self, instance_id: str, tp_rank: int, device_id: int, load_state_shm: str,
             layer_names: Sequence[str], block_ids: Sequence[int], block_hashes: Sequence[bytes]) -> tuple[bool, str]:
        req = P.LoadRequest(instance_id=instance_id, tp_rank=tp_rank, device_id=device_id,
                            load_state_shm=load_state_shm, layer_names=list(layer_names), block_ids=list(block_ids),
                            block_hashes=list(block_hashes))
        return self._status("load", self._call("Load", req))

    def query(self, instance_id: str, block_hashes: Sequence[bytes]) -> dict:
        r = self._call("Query", P.QueryRequest(instance_id=instance_id, block_hashes=list(block_hashes)))
        ok, msg = self._status("query", r)
        return {"ok": ok, "message": msg, "hit_blocks": r.hit_blocks,
                "prefetch_state": _PREFETCH.get(r.prefetch_state, "ready"), "loading_blocks": r.loading_blocks,
                "missing_blocks": r.missing_blocks}

    def unregister_context(self, instance_id: str) -> tuple[bool, str]:
        return self._status("unregister_context",
                            self._call("UnregisterContext", P.UnregisterRequest(instance_id=instance_id)))

    def shutdown(self) -> tuple[bool, str]:
        return self._status("shutdown", self._call("Shutdown", P.ShutdownRequest()))

    def close(self) -> None:
        self._channel.close()
