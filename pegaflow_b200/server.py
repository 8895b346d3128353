"""gRPC ``pegaflow.Engine`` server over the B200 engine.

Restates the reference server (pegaflow-server/src): the seven RPCs of
engine.proto on the same wire schema (pegaflow_b200.proto), the EngineError ->
gRPC status mapping (service.rs:77-88), the CUDA IPC tensor registry that
keeps the vLLM workers' KV tensors mapped in this process (registry.rs), and
the command line (lib.rs:43-113). Run with ``python -m pegaflow_b200.server``.

The DFS tier (seal_offload.rs) is served by --dfs-local-index: packed files
under --dfs-root in the reference's format, with the block metadata in
sidecar files, since this build has no Redis (--redis-url is refused). OTel
export is not served (its flags are accepted).
"""

from __future__ import annotations

import argparse
import logging
import threading
from concurrent import futures
from typing import Callable, Optional

import grpc

from . import proto as P

log = logging.getLogger("pegaflow_b200.server")

DEFAULT_ADDR = "127.0.0.1:50055"
DRAIN_TIMEOUT_S = 60.0  # how long teardown waits for copies that use mapped tensors


def parse_memory_size(s: str) -> int:
    """Size with an optional kb/mb/gb/tb suffix (pegaflow-server/src/utils.rs:3-34)."""
    s = s.strip()
    boundary = next((i for i, c in enumerate(s) if c.isascii() and c.isalpha()), len(s))
    num, unit = s[:boundary], s[boundary:]
    try:
        value = float(num.strip())
    except ValueError:
        raise ValueError(f"Invalid number: '{num}'") from None
    if value < 0:
        raise ValueError("Memory size cannot be negative")
    unit = unit.strip().lower()
    mult = {"": 1, "b": 1, "kb": 1 << 10, "mb": 1 << 20, "gb": 1 << 30, "tb": 1 << 40}.get(unit)
    if mult is None:
        raise ValueError(f"Unknown unit: '{unit}'. Use kb, mb, gb, or tb")
    return int(value * mult)


class TensorRegistry:
    """KV tensors mapped from the workers' CUDA IPC handles, kept alive per
    context "{instance}:tp{rank}:dev{device}" (registry.rs:30-175)."""

    def __init__(self, materialize: Optional[Callable[[int, bytes], tuple]] = None):
        self._materialize = materialize or self._from_ipc
        self._contexts: dict[str, dict] = {}
        self._lock = threading.Lock()

    @staticmethod
    def _from_ipc(device_id: int, wrapper_bytes: bytes):
        import torch

        from .ipc import loads_wrapper

        torch.cuda.set_device(device_id)
        tensor = loads_wrapper(wrapper_bytes).to_tensor()
        device = tensor.device.index if tensor.device.index is not None else device_id
        return tensor, tensor.data_ptr(), tensor.untyped_storage().nbytes(), device

    def register_layer(self, context_key: str, layer_name: str, device_id: int, wrapper_bytes: bytes):
        keep, data_ptr, size_bytes, device = self._materialize(device_id, wrapper_bytes)
        with self._lock:
            ctx = self._contexts.setdefault(context_key, {"device": device, "tensors": {}})
            if ctx["device"] != device:
                raise ValueError(f"context {context_key} is pinned to device {ctx['device']} but got {device}")
            ctx["tensors"][layer_name] = keep
        return data_ptr, size_bytes, device

    def devices_of(self, instance_id: str) -> set:
        prefix = f"{instance_id}:"
        with self._lock:
            return {c["device"] for k, c in self._contexts.items() if k.startswith(prefix)}

    def all_devices(self) -> set:
        with self._lock:
            return {c["device"] for c in self._contexts.values()}

    def drop_instance(self, instance_id: str) -> int:
        prefix = f"{instance_id}:"
        with self._lock:
            keys = [k for k in self._contexts if k.startswith(prefix)]
            count = sum(len(self._contexts[k]["tensors"]) for k in keys)
            for k in keys:
                del self._contexts[k]
        return count

    def clear(self) -> None:
        with self._lock:
            self._contexts.clear()


def _status_code(err) -> grpc.StatusCode:
    """EngineError -> gRPC code (service.rs:77-88)."""
    from . import _native as N

    code = getattr(err, "code", None)
    if code == N.PF_ERR_INVALID_ARGUMENT:
        return grpc.StatusCode.INVALID_ARGUMENT
    if code in (N.PF_ERR_INSTANCE_MISSING, N.PF_ERR_WORKER_MISSING, N.PF_ERR_TOPOLOGY_MISMATCH):
        return grpc.StatusCode.FAILED_PRECONDITION
    return grpc.StatusCode.INTERNAL


class EngineService:
    """Handlers of service pegaflow.Engine (service.rs:133-405)."""

    def __init__(self, engine, registry: Optional[TensorRegistry] = None, on_shutdown: Optional[Callable] = None):
        self.engine = engine
        self.registry = registry or TensorRegistry()
        self.on_shutdown = on_shutdown
        self._busy: dict[str, int] = {}  # instance -> Save/Load RPCs running
        self._busy_cv = threading.Condition()

    def _tracked(self, instance_id: str, context, fn, *args):
        """An engine call that reads or writes the instance's mapped tensors."""
        with self._busy_cv:
            self._busy[instance_id] = self._busy.get(instance_id, 0) + 1
        try:
            return self._engine_call(context, fn, *args)
        finally:
            with self._busy_cv:
                self._busy[instance_id] -= 1
                if not self._busy[instance_id]:
                    del self._busy[instance_id]
                self._busy_cv.notify_all()

    def _drain(self, instance_id: Optional[str], devices) -> None:
        """Wait for running Save/Load RPCs (of one instance, or all) and for
        the loads queued on `devices`, so the tensors can be unmapped."""
        with self._busy_cv:
            done = self._busy_cv.wait_for(
                lambda: (instance_id not in self._busy) if instance_id else not self._busy, timeout=DRAIN_TIMEOUT_S)
        if not done:
            log.warning("RPCs still running after %.0f s; unmapping anyway", DRAIN_TIMEOUT_S)
        for d in sorted(devices):
            try:
                self.engine.wait_loads(d, DRAIN_TIMEOUT_S)
            except Exception as e:
                log.warning("loads on device %d did not finish: %s", d, e)

    @staticmethod
    def _ok():
        return P.ResponseStatus(ok=True, message="")

    def _engine_call(self, context, fn, *args):
        from ._native import PegaError

        try:
            return fn(*args)
        except PegaError as e:
            context.abort(_status_code(e), str(e))

    def RegisterContext(self, req, context):
        try:
            data_ptr, size_bytes, device = self.registry.register_layer(
                f"{req.instance_id}:tp{req.tp_rank}:dev{req.device_id}", req.layer_name, req.device_id,
                req.wrapper_bytes)
        except Exception as e:  # map_py_error (service.rs:90-93)
            context.abort(grpc.StatusCode.INTERNAL, f"register tensor failed: {e}")
        self._engine_call(context, self.engine.register_context_layer, req.instance_id, req.namespace, device,
                          req.layer_name, data_ptr, size_bytes, req.num_blocks, req.bytes_per_block,
                          req.kv_stride_bytes, req.segments, req.tp_rank, req.tp_size, req.num_layers)
        return P.RegisterContextResponse(status=self._ok())

    # Save and Load carry the data path's block lists: a Save for 80 layers x
    # 2,048 blocks is about 6 MB of ids and hashes. Their wire bytes go to the
    # library, which decodes them natively (csrc/wire.cpp) with the GIL
    # released, instead of building per-layer Python lists.
    RAW_REQUESTS = ("Save", "Load")

    def Save(self, raw: bytes, context):
        from .engine import request_instance_id

        instance_id = self._engine_call(context, request_instance_id, raw)
        self._tracked(instance_id, context, self.engine.save_request, raw)
        return P.SaveResponse(status=self._ok())

    def Load(self, raw: bytes, context):
        from .engine import request_instance_id

        instance_id = self._engine_call(context, request_instance_id, raw)
        self._tracked(instance_id, context, self.engine.load_request, raw)
        return P.LoadResponse(status=self._ok())

    def Query(self, req, context):
        # service.rs:262-319: with the packed-file tier on, a prefix that the
        # tier holds is read back in the background and reported as LOADING.
        q = self._engine_call(context, self.engine.query_prefetch, req.instance_id, list(req.block_hashes))
        state = {"ready": P.PREFETCH_READY, "loading": P.PREFETCH_LOADING,
                 "partial_miss": P.PREFETCH_PARTIAL_MISS}[q["prefetch_state"]]
        return P.QueryResponse(status=self._ok(), hit_blocks=q["hit_blocks"], prefetch_state=state,
                               loading_blocks=q["loading_blocks"], missing_blocks=q["missing_blocks"])

    def UnregisterContext(self, req, context):
        # The reference drops the mapped KV tensors first (service.rs:340-353).
        # Here the engine forgets the instance first, so no new copy starts.
        # Then RPCs already running for it and loads queued on its devices
        # finish, and only then are the tensors unmapped: a copy never touches
        # a closed mapping. The engine's error, if any, is still returned.
        from ._native import PegaError

        err = None
        try:
            self.engine.unregister_instance(req.instance_id)
        except PegaError as e:
            err = e
        self._drain(req.instance_id, self.registry.devices_of(req.instance_id))
        dropped = self.registry.drop_instance(req.instance_id)
        if dropped:
            log.info("Dropped %d CUDA tensors for instance %s", dropped, req.instance_id)
        if err is not None:
            context.abort(_status_code(err), str(err))
        return P.UnregisterResponse(status=self._ok())

    def Shutdown(self, req, context):
        self._drain(None, self.registry.all_devices())
        self.registry.clear()
        log.warning("Shutdown requested via RPC")
        if self.on_shutdown:
            threading.Thread(target=self.on_shutdown, daemon=True).start()
        return P.ShutdownResponse(status=self._ok())

    def Health(self, req, context):
        return P.HealthResponse(status=self._ok())

    def handler(self) -> grpc.GenericRpcHandler:
        methods = {}
        for rpc, (req_name, resp_name) in P.METHODS.items():
            methods[rpc] = grpc.unary_unary_rpc_method_handler(
                getattr(self, rpc),
                request_deserializer=None if rpc in self.RAW_REQUESTS else P.M[req_name].FromString,
                response_serializer=P.M[resp_name].SerializeToString)
        return grpc.method_handlers_generic_handler(P.SERVICE, methods)


def serve(engine, addr: str = DEFAULT_ADDR, registry: Optional[TensorRegistry] = None, max_workers: int = 32):
    """Start the service on `addr`; returns (server, service, bound port)."""
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers),
                         options=[("grpc.max_receive_message_length", 256 << 20),
                                  ("grpc.max_send_message_length", 256 << 20)])
    service = EngineService(engine, registry, on_shutdown=lambda: server.stop(grace=1.0))
    server.add_generic_rpc_handlers((service.handler(),))
    port = server.add_insecure_port(addr)
    if port == 0:
        raise RuntimeError(f"cannot bind {addr}")
    server.start()
    return server, service, port


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="pegaflow_b200.server",
                                 description="PegaEngine gRPC server with CUDA IPC registry (B200 engine)")
    ap.add_argument("--addr", default=DEFAULT_ADDR)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--pool-size", type=parse_memory_size, default=parse_memory_size("30gb"))
    ap.add_argument("--hint-value-size", type=parse_memory_size, default=None)
    ap.add_argument("--use-hugepages", action="store_true")
    ap.add_argument("--pre-evict", action="store_true")
    ap.add_argument("--pre-evict-threshold", type=parse_memory_size, default=parse_memory_size("5gb"))
    ap.add_argument("--pre-evict-target", type=parse_memory_size, default=parse_memory_size("8gb"))
    ap.add_argument("--pre-evict-interval-ms", type=int, default=100)
    ap.add_argument("--disable-lfu-admission", action="store_true")
    ap.add_argument("--numa-pools", choices=["off", "node", "device"], default="off",
                    help="split the pool per NUMA node of the GPUs (or per GPU), each part on its GPUs' node; "
                         "a save allocates from its GPU's part (not a reference flag)")
    ap.add_argument("--metrics-otel-endpoint", default="http://127.0.0.1:4321")
    ap.add_argument("--metrics-period-secs", type=int, default=5)
    ap.add_argument("--log-level", default="info")
    ap.add_argument("--redis-url", default=None)
    ap.add_argument("--dfs-root", default="/tmp/pega")
    ap.add_argument("--dfs-quota", type=parse_memory_size, default=parse_memory_size("50gb"))
    ap.add_argument("--dfs-scan-interval-ms", type=int, default=100)
    ap.add_argument("--dfs-local-index", action="store_true",
                    help="write sealed blocks through to packed files under --dfs-root and prefetch them back "
                         "on a query miss, with the block metadata in sidecar files instead of Redis")
    return ap


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    logging.basicConfig(level=getattr(logging, args.log_level.upper(), logging.INFO),
                        format="%(asctime)s %(levelname)s %(name)s: %(message)s")
    if args.redis_url:
        raise SystemExit("--redis-url: block metadata is not kept in Redis by this build; "
                         "--dfs-local-index keeps it in sidecar files under --dfs-root")
    import torch

    if torch.cuda.is_available():
        torch.cuda.init()
        torch.cuda.set_device(args.device)
    from .engine import PegaEngine

    pre_evict = (args.pre_evict_threshold, args.pre_evict_target, args.pre_evict_interval_ms) if args.pre_evict else None
    dfs = dict(dfs_root=args.dfs_root, dfs_quota=args.dfs_quota,
               dfs_scan_interval_ms=args.dfs_scan_interval_ms) if args.dfs_local_index else {}
    engine = PegaEngine(args.pool_size, args.use_hugepages, enable_lfu_admission=not args.disable_lfu_admission,
                        hint_value_size_bytes=args.hint_value_size or 0, pre_evict=pre_evict,
                        numa_pools=args.numa_pools, **dfs)
    server, _, port = serve(engine, args.addr)
    log.info("pegaflow_b200 engine server listening on %s (port %d)", args.addr, port)
    server.wait_for_termination()
    engine.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
