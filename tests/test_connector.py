"""The vLLM connector against fixtures recorded from the reference's own
connector code (tests/golden/, made by make_golden.py): request-tracker
traces, namespace derivation, registration arguments, save-batch and load RPC
composition. CPU only; the engine client is a recording fake."""

import json
import types
from pathlib import Path

import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


class Recorder:
    def __init__(self):
        self.calls = []

    def register_context(self, *a):
        self.calls.append(("register_context", a))
        return True, ""

    def save(self, *a):
        self.calls.append(("save", a))
        return True, ""

    def load(self, *a):
        self.calls.append(("load", a))
        return True, ""

    def unregister_context(self, *a):
        self.calls.append(("unregister_context", a))
        return True, ""

    def query(self, instance_id, hashes):
        self.calls.append(("query", (instance_id, hashes)))
        return {"ok": True, "message": "", "hit_blocks": self.hits, "prefetch_state": "ready", "loading_blocks": 0,
                "missing_blocks": 0}


class FakeState:
    def __init__(self, n=0):
        self.n = n

    def shm_name(self):
        return "pega_load_golden"

    def is_ready(self):
        return False


def ctx(client, num_layers=3, layerwise=False):
    from pegaflow_b200.connector import ConnectorContext

    return ConnectorContext("inst", "ns", 16, num_layers, 1, 0, 0, client, layerwise)


def test_request_tracker_matches_reference_traces():
    from pegaflow_b200.connector import RequestTracker

    traces = json.loads((GOLDEN / "tracker_traces.json").read_text())
    assert len(traces) == 40
    for tr in traces:
        t = RequestTracker("r", [bytes.fromhex(h) for h in tr["hashes"]], tr["block_size"], tr["layers"])
        for (op, args), (expect, phase, done) in zip(tr["ops"], tr["outs"]):
            out = None
            if op == "lookup":
                t.on_lookup(*args)
            elif op == "alloc":
                t.on_alloc(*args)
            elif op == "load":
                li = t.consume_load_intent()
                out = None if li is None else [list(li.block_ids), [h.hex() for h in li.block_hashes], li.num_tokens]
            elif op == "sched":
                t.on_scheduled(*args)
            elif op == "save":
                si = t.consume_save_intent()
                out = None if si is None else [list(si.block_ids), [h.hex() for h in si.block_hashes]]
            elif op == "layer":
                t.on_layer_saved()
            elif op == "finish":
                t.on_finished()
            else:
                out = t.should_hold_blocks()
            assert [out, t.phase.value, t.is_done()] == [expect, phase, done], (tr["ops"], op)


def test_namespace_matches_reference():
    from pegaflow_b200.connector import namespace_from_factors

    g = json.loads((GOLDEN / "namespace.json").read_text())
    assert namespace_from_factors(g["factors"]) == g["namespace"]


def test_registration_arguments_match_reference():
    import torch

    from pegaflow_b200.connector import WorkerSide

    dtypes = {1: torch.uint8, 2: torch.bfloat16, 4: torch.float32}
    for case in json.loads((GOLDEN / "registration.json").read_text()):
        rec = Recorder()
        w = WorkerSide(ctx(rec, num_layers=1), wrapper_factory=lambda t: b"wrapper")
        try:
            w.register_kv_caches({case["case"]: torch.empty(case["shape"], dtype=dtypes[case["element_size"]],
                                                            device="meta")})
        finally:
            w._save_q.put(None)
            w._save_thread.join()
        (_, args), = rec.calls
        assert list(args[8:12]) == [case["num_blocks"], case["bytes_per_block"], case["kv_stride_bytes"],
                                    case["segments"]], case["case"]
        assert args[:7] == ("inst", "ns", 0, 1, 0, 1, case["case"])


def test_token_major_registration_matches_reference_sglang_adapter():
    """configs[0] registers separate K and V buffers as segments=1 layers, as
    the reference's SGLang adapter does; its registration arguments for
    token-major buffers were recorded by make_golden.py."""
    import torch

    from pegaflow_b200 import Layout

    dtypes = {2: torch.float16, 4: torch.float32}
    for case in json.loads((GOLDEN / "sglang_registration.json").read_text()):
        t = torch.empty(case["shape"], dtype=dtypes[case["element_size"]], device="meta")
        lay = Layout.from_token_major(t, case["page_size"])
        assert (lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, lay.segments) == (
            case["num_blocks"], case["bytes_per_block"], case["kv_stride_bytes"], case["segments"]), case["case"]
        assert case["num_layers"] == 24
    # The same memory seen as vLLM-style blocks [blocks, page, heads, dim]
    # registers identically (the GPT-2 shape of configs[0]).
    t = torch.empty((4096, 12, 64), dtype=torch.float16, device="meta")
    a, b = Layout.from_token_major(t, 16), Layout.from_tensor(t.view(256, 16, 12, 64))
    assert (a.num_blocks, a.bytes_per_block, a.segments) == (b.num_blocks, b.bytes_per_block, b.segments)


def _meta(intents):
    from pegaflow_b200.connector import PegaConnectorMetadata, SaveIntent

    return PegaConnectorMetadata(save_intents={
        k: SaveIntent(tuple(v["block_ids"]), tuple(bytes.fromhex(h) for h in v["block_hashes"]))
        for k, v in intents.items()})


def test_save_batch_rpc_matches_reference():
    from pegaflow_b200.connector.worker import WorkerSide, _SaveTask

    g = json.loads((GOLDEN / "save_batches.json").read_text())
    rec = Recorder()
    w = WorkerSide(ctx(rec))
    meta = _meta(g["save_intents"])
    tasks = [_SaveTask(t["layer"], types.SimpleNamespace(block_table=object() if t["has_block_table"] else None),
                       meta, ["reqA", "reqB", "reqC"] if i < 3 else ["reqA"])
             for i, t in enumerate(g["tasks"])]
    w.process_save_batch(tasks)
    w._save_q.put(None)
    w._save_thread.join()
    saves = [a for n, a in rec.calls if n == "save"]
    assert len(saves) == len(g["rpc"]) == 1
    (inst, rank, dev, layers), want = saves[0], g["rpc"][0]
    assert (inst, rank, dev) == (want["instance_id"], want["tp_rank"], want["device_id"])
    assert [[n, list(ids), [h.hex() for h in hs]] for n, ids, hs in layers] == want["saves"]


def test_load_rpc_matches_reference():
    from pegaflow_b200.connector import LoadIntent, PegaConnectorMetadata, SaveIntent, WorkerSide

    g = json.loads((GOLDEN / "load_requests.json").read_text())
    rec = Recorder()
    w = WorkerSide(ctx(rec), load_state_factory=FakeState)
    meta = PegaConnectorMetadata(
        load_intents={k: LoadIntent(tuple(v["block_ids"]), tuple(bytes.fromhex(h) for h in v["block_hashes"]),
                                    16 * len(v["block_ids"])) for k, v in g["load_intents"].items()},
        save_intents={"r3": SaveIntent((1,), (b"q",))})
    layers = {k: (types.SimpleNamespace(kv_cache=[None]) if v else types.SimpleNamespace())
              for k, v in g["layers"].items()}
    w.start_load_kv(meta, types.SimpleNamespace(no_compile_layers=layers))
    w._save_q.put(None)
    w._save_thread.join()
    (_, args), = [c for c in rec.calls if c[0] == "load"]
    (want,) = g["rpc"]
    assert args[0:3] == (want["instance_id"], want["tp_rank"], want["device_id"])
    assert list(args[4]) == want["layer_names"] and list(args[5]) == want["block_ids"]
    assert [h.hex() for h in args[6]] == want["block_hashes"]


def test_shutdown_sends_queued_saves_before_unregistering():
    import threading

    from pegaflow_b200.connector import WorkerSide

    release, entered = threading.Event(), threading.Event()

    class SlowSaves(Recorder):
        def save(self, *a):
            entered.set()
            release.wait(10)
            return super().save(*a)

    rec = SlowSaves()
    w = WorkerSide(ctx(rec, num_layers=1), wrapper_factory=lambda t: b"w")
    w._layers = ["L0"]  # registered
    meta = _meta({"r1": {"block_ids": [1, 2], "block_hashes": ["aa", "bb"]}})
    w.save_kv_layer(meta, "L0", None, types.SimpleNamespace(block_table=object()))
    assert entered.wait(10)  # the save is in flight
    stopper = threading.Thread(target=w.shutdown)
    stopper.start()
    stopper.join(0.2)  # shutdown must wait for it, not unregister meanwhile
    release.set()
    stopper.join(10)
    assert [name for name, _ in rec.calls] == ["save", "unregister_context"]


def test_scheduler_flow_async_and_layerwise():
    from pegaflow_b200.connector import SchedulerSide

    for layerwise in (False, True):
        rec = Recorder()
        rec.hits = 3
        s = SchedulerSide(ctx(rec, layerwise=layerwise))
        req = types.SimpleNamespace(request_id="r", block_hashes=[b"a", b"b", b"c", b"d"], num_tokens=64)
        tokens, is_async = s.get_num_new_matched_tokens(req, 16)
        assert tokens == 32 and is_async is (not layerwise)  # 3 hit blocks, 1 already computed
        blocks = types.SimpleNamespace(get_block_ids=lambda: ([7, 8, 9, 10],))
        s.update_state_after_alloc(req, blocks, 32)
        out = types.SimpleNamespace(scheduled_new_reqs=[types.SimpleNamespace(req_id="r")],
                                    num_scheduled_tokens={"r": 64},
                                    scheduled_cached_reqs=types.SimpleNamespace(req_ids=[], new_block_ids=[]))
        meta = s.build_connector_meta(out)
        assert meta.load_intents["r"].block_ids == (8, 9) and meta.load_intents["r"].num_tokens == 32
        assert meta.save_intents["r"].block_ids == (7, 8, 9, 10)
        assert s.request_finished(req, [])[0] is True  # blocks held until the save lands
        s.update_connector_output(types.SimpleNamespace(finished_sending={"r"}))
        assert "r" not in s._trackers
