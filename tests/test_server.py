"""gRPC surface on CPU: engine.proto wire format, the reference's CLI size
parser tests (pegaflow-server/src/utils.rs:38-58), server + EngineRpcClient
round trips over a host-memory engine, status-code mapping (service.rs:77-88)
and the restricted unpickling of IPC wrapper bytes."""

import pickle
import sys
import types

import pytest


# ------------------------------------------------------------------ size parser


def test_parse_memory_size_basic():
    from pegaflow_b200.server import parse_memory_size

    assert parse_memory_size("1024") == 1024
    assert parse_memory_size("1gb") == 1024**3
    assert parse_memory_size("1.5gb") == int(1.5 * 1024**3)
    assert parse_memory_size("500MB") == 500 << 20
    assert parse_memory_size(" 2 tb ") == 2 << 40


def test_server_flags():
    """The reference server's flags (pegaflow-server/src/lib.rs:43-113) plus
    --numa-pools, with their defaults."""
    from pegaflow_b200.server import build_parser

    a = build_parser().parse_args([])
    assert (a.pool_size, a.numa_pools, a.disable_lfu_admission, a.dfs_local_index) == (30 << 30, "off", False, False)
    a = build_parser().parse_args(["--pool-size", "2gb", "--numa-pools", "device", "--pre-evict",
                                   "--dfs-local-index", "--dfs-root", "/x", "--dfs-quota", "1gb"])
    assert (a.pool_size, a.numa_pools, a.pre_evict, a.dfs_root, a.dfs_quota) == (2 << 30, "device", True, "/x",
                                                                                  1 << 30)
    with pytest.raises(SystemExit):
        build_parser().parse_args(["--numa-pools", "socket"])


def test_parse_memory_size_invalid():
    from pegaflow_b200.server import parse_memory_size

    for bad in ["", "abc", "-10gb", "10pb"]:
        with pytest.raises(ValueError):
            parse_memory_size(bad)


# ------------------------------------------------------------------ wire format


def test_proto_wire_bytes():
    """Hand-checked protobuf encodings of engine.proto messages (field numbers
    and types engine.proto:5-105)."""
    from pegaflow_b200 import proto as P

    r = P.SaveRequest(instance_id="i", tp_rank=1, device_id=-1,
                      saves=[P.SaveLayer(layer_name="L", block_ids=[1, 2, 300], block_hashes=[b"ab"])])
    assert r.SerializeToString().hex() == (
        "0a0169" "1001" "18ffffffffffffffffff01" "220d" "0a014c" "12040102ac02" "1a026162")
    q = P.QueryResponse(status=P.ResponseStatus(ok=True), hit_blocks=5, prefetch_state=P.PREFETCH_LOADING)
    assert q.SerializeToString().hex() == "0a0208011005" "1801"
    reg = P.RegisterContextRequest(namespace="n", num_layers=3)
    assert reg.SerializeToString().hex() == "5803" "62016e"
    assert set(P.METHODS) == {"RegisterContext", "Save", "Load", "Query", "UnregisterContext", "Shutdown", "Health"}


# ------------------------------------------------------------------ server round trip


@pytest.fixture
def served(native):
    import numpy as np

    from pegaflow_b200 import EngineRpcClient, PegaEngine
    from pegaflow_b200.server import TensorRegistry, serve

    engine = PegaEngine(1 << 20, pool_kind="host")
    fake = np.zeros(2 * 16 * 4096, np.uint8)

    def materialize(device_id, wrapper_bytes):
        assert wrapper_bytes == b"wrapper"
        return fake, fake.ctypes.data, fake.nbytes, device_id

    server, service, port = serve(engine, "127.0.0.1:0", TensorRegistry(materialize))
    client = EngineRpcClient(f"http://127.0.0.1:{port}", connect_timeout_s=5)
    yield client, service, engine
    client.close()
    server.stop(0)
    engine.close()


def test_health_register_query_unregister(served):
    client, service, engine = served
    assert client.health() == (True, "")
    assert client.endpoint().startswith("http://127.0.0.1:")
    ok, msg = client.register_context("inst", "ns", 0, 1, 0, 2, "L0", b"wrapper", 16, 4096, 16 * 4096, 2)
    assert (ok, msg) == (True, "")
    r = client.query("inst", [b"a", b"b"])
    assert r == {"ok": True, "message": "", "hit_blocks": 0, "prefetch_state": "ready", "loading_blocks": 0,
                 "missing_blocks": 0}
    assert client.unregister_context("inst") == (True, "")
    assert service.registry.drop_instance("inst") == 0


def test_query_reports_packed_file_tier_states(native, tmp_path):
    """With the packed-file tier on, Query carries the tier's state
    (service.rs:283-305): blocks held nowhere are a partial miss."""
    import numpy as np

    from pegaflow_b200 import EngineRpcClient, PegaEngine
    from pegaflow_b200.server import TensorRegistry, serve

    engine = PegaEngine(1 << 20, pool_kind="host", dfs_root=str(tmp_path / "dfs"))
    fake = np.zeros(2 * 16 * 4096, np.uint8)
    server, _, port = serve(engine, "127.0.0.1:0",
                            TensorRegistry(lambda d, w: (fake, fake.ctypes.data, fake.nbytes, d)))
    client = EngineRpcClient(f"http://127.0.0.1:{port}", connect_timeout_s=5)
    try:
        client.register_context("inst", "ns", 0, 1, 0, 1, "L0", b"w", 16, 4096, 16 * 4096, 2)
        r = client.query("inst", [b"a", b"b", b"c"])
        assert (r["prefetch_state"], r["hit_blocks"], r["missing_blocks"]) == ("partial_miss", 0, 3)
    finally:
        client.close()
        server.stop(0)
        engine.close()


def test_unregister_unmaps_tensors_only_after_copies_that_use_them(native):
    """A Save RPC still copying from an instance's KV tensors, and loads
    queued on its devices, finish before UnregisterContext unmaps them."""
    import threading
    import time

    from pegaflow_b200 import proto as P

    from pegaflow_b200.server import EngineService, TensorRegistry

    events, in_save, release = [], threading.Event(), threading.Event()

    class Engine:
        def register_context_layer(self, *a):
            events.append("register")

        def save_request(self, raw):
            assert P.SaveRequest.FromString(raw).instance_id == "i"
            in_save.set()
            release.wait(10)
            events.append("save done")

        def unregister_instance(self, instance_id):
            events.append("unregister")

        def wait_loads(self, device_id, timeout_s):
            events.append(f"wait_loads {device_id}")

    class Registry(TensorRegistry):
        def drop_instance(self, instance_id):
            events.append("drop")
            return super().drop_instance(instance_id)

    svc = EngineService(Engine(), Registry(lambda d, w: (object(), 0x1000, 4096, d)))

    def abort(code, msg):
        raise RuntimeError(msg)

    ctx = types.SimpleNamespace(abort=abort)
    svc.RegisterContext(types.SimpleNamespace(instance_id="i", tp_rank=0, device_id=3, layer_name="L0",
                                              wrapper_bytes=b"w", namespace="ns", num_blocks=1,
                                              bytes_per_block=4096, kv_stride_bytes=0, segments=1, tp_size=1,
                                              num_layers=1), ctx)
    save = threading.Thread(target=svc.Save,
                            args=(P.SaveRequest(instance_id="i", tp_rank=0, device_id=3).SerializeToString(), ctx))
    save.start()
    assert in_save.wait(5)
    unreg = threading.Thread(target=svc.UnregisterContext, args=(types.SimpleNamespace(instance_id="i"), ctx))
    unreg.start()
    time.sleep(0.2)
    assert "drop" not in events  # waiting for the save that reads the tensors
    release.set()
    save.join(5)
    unreg.join(5)
    assert events == ["register", "unregister", "save done", "wait_loads 3", "drop"]


def test_errors_become_grpc_status_codes(served):
    client, _, _ = served
    client.register_context("inst", "ns", 0, 1, 0, 2, "L0", b"wrapper", 16, 4096, 16 * 4096, 2)
    with pytest.raises(RuntimeError, match="INVALID_ARGUMENT.*block_ids length 2 does not match block_hashes 1"):
        client.save("inst", 0, 0, [("L0", [1, 2], [b"x"])])
    with pytest.raises(RuntimeError, match="FAILED_PRECONDITION.*instance nope not found"):
        client.query("nope", [b"a"])
    with pytest.raises(RuntimeError, match="FAILED_PRECONDITION.*topology mismatch"):
        client.register_context("inst", "ns", 0, 4, 0, 2, "L1", b"wrapper", 16, 4096, 16 * 4096, 2)
    with pytest.raises(RuntimeError, match="INTERNAL.*register tensor failed"):
        client.register_context("inst", "ns", 0, 1, 0, 2, "L1", b"bad", 16, 4096, 16 * 4096, 2)
    from pegaflow_b200 import PyLoadState

    s = PyLoadState()
    with pytest.raises(RuntimeError, match="INTERNAL.*missing KV block hash at index 0"):
        client.load("inst", 0, 0, s.shm_name(), ["L0"], [1], [b"zz"])
    assert s.get_state() == -1


def test_save_of_negative_ids_and_shutdown(served):
    client, _, _ = served
    client.register_context("inst", "ns", 0, 1, 0, 2, "L0", b"wrapper", 16, 4096, 16 * 4096, 2)
    assert client.save("inst", 0, 0, [("L0", [-1], [b"x"])]) == (True, "")
    assert client.shutdown() == (True, "")


def test_client_connect_timeout():
    from pegaflow_b200 import EngineRpcClient

    with pytest.raises(RuntimeError, match="failed to connect to engine server at http://127.0.0.1:1"):
        EngineRpcClient("http://127.0.0.1:1", connect_timeout_s=0.2)


# ------------------------------------------------------------------ wrapper unpickling


def _reference_style_wrapper_bytes(**attrs) -> bytes:
    """Pickle an object whose class lives at the reference's path
    pegaflow.ipc_wrapper.CudaIPCWrapper, as the reference worker does."""
    mod = types.ModuleType("pegaflow.ipc_wrapper")

    class CudaIPCWrapper:
        pass

    CudaIPCWrapper.__module__ = "pegaflow.ipc_wrapper"
    CudaIPCWrapper.__qualname__ = "CudaIPCWrapper"
    mod.CudaIPCWrapper = CudaIPCWrapper
    pkg = types.ModuleType("pegaflow")
    saved = {k: sys.modules.get(k) for k in ("pegaflow", "pegaflow.ipc_wrapper")}
    sys.modules["pegaflow"], sys.modules["pegaflow.ipc_wrapper"] = pkg, mod
    try:
        w = CudaIPCWrapper()
        w.__dict__.update(attrs)
        return pickle.dumps(w)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def test_reference_wrapper_bytes_load_into_our_class():
    import torch

    from pegaflow_b200.ipc import CudaIPCWrapper, loads_wrapper

    data = _reference_style_wrapper_bytes(handle=(0, b"\x01" * 64, 4096, 0, b"ref", 7, b"ev", False),
                                          dtype=torch.bfloat16, shape=torch.Size([2, 16, 8]), device_uuid="GPU-x")
    w = loads_wrapper(data)
    assert isinstance(w, CudaIPCWrapper)
    assert w.dtype == torch.bfloat16 and tuple(w.shape) == (2, 16, 8) and w.device_uuid == "GPU-x"


def test_wrapper_unpickling_refuses_other_globals():
    from pegaflow_b200.ipc import loads_wrapper

    evil = pickle.dumps(types.SimpleNamespace(x=1))
    with pytest.raises(pickle.UnpicklingError, match="may not reference"):
        loads_wrapper(evil)
    with pytest.raises(pickle.UnpicklingError, match="not a CudaIPCWrapper"):
        loads_wrapper(pickle.dumps({"a": 1}))
    # A call smuggled in as a reduce of an allowed-looking name is refused too.
    with pytest.raises(pickle.UnpicklingError, match="may not reference os.system"):
        loads_wrapper(b"cos\nsystem\n(S'true'\ntR.")
    # Old pickle protocols rebuild objects through copyreg, which is not allowed.
    import torch

    from pegaflow_b200.ipc import CudaIPCWrapper

    w = CudaIPCWrapper.__new__(CudaIPCWrapper)
    w.handle, w.dtype, w.shape, w.device_uuid = (0,), torch.float16, torch.Size([1]), "GPU-x"
    with pytest.raises(pickle.UnpicklingError, match="_reconstructor"):
        loads_wrapper(pickle.dumps(w, protocol=0))
