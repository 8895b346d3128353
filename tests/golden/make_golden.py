"""Generate golden fixtures from the reference's own Python connector code.

Runs the reference's vLLM worker connector (python/pegaflow/connector/worker.py
in the xiaguan/pegaflow tree) with its Rust extension and CUDA IPC wrapper
replaced by recording stubs, and records what it sends to the engine:

  * registration.json — register_context(...) arguments the worker derives
    from KV tensors of the benchmark shapes (worker.py:80-146);
  * save_batches.json — the (layer, block_ids, block_hashes) list one save
    RPC carries for a batch of per-layer save tasks (worker.py:372-427);
  * load_requests.json — the load RPC arguments of start_load_kv
    (worker.py:217-286);
  * tracker_traces.json, namespace.json — request-tracker traces and the
    namespace hash (connector/common.py);
  * sglang_registration.json — register_context arguments of the SGLang
    adapter for token-major K/V buffers (sglang/peagflow_radix_cache.py:
    160-250), with sglang's own modules stubbed.

Usage (needs the reference tree; not run by the test suite):
    python tests/golden/make_golden.py /path/to/pegaflow
"""

from __future__ import annotations

import json
import sys
import types
from pathlib import Path

import torch

OUT = Path(__file__).resolve().parent


class _Recorder:
    calls: list = []


class FakeEngineRpcClient:
    def __init__(self, endpoint=None):
        self.endpoint = endpoint

    def register_context(self, *args):
        _Recorder.calls.append(("register_context", args))
        return True, ""

    def save(self, *args):
        _Recorder.calls.append(("save", args))
        return True, ""

    def load(self, *args):
        _Recorder.calls.append(("load", args))
        return True, ""

    def query(self, *args):
        return {"ok": True, "message": "", "hit_blocks": 0, "prefetch_state": "ready", "loading_blocks": 0,
                "missing_blocks": 0}

    def unregister_context(self, *args):
        return True, ""


class FakeLoadState:
    def shm_name(self):
        return "pega_load_golden"

    def get_state(self):
        return 0

    def is_ready(self):
        return False


class CudaIPCWrapper:  # picklable stand-in for pegaflow.ipc_wrapper.CudaIPCWrapper
    def __init__(self, tensor):
        self.shape = tuple(tensor.shape)


def install_stubs(ref_python: Path) -> None:
    ext = types.ModuleType("pegaflow.pegaflow")
    ext.EngineRpcClient = FakeEngineRpcClient
    ext.PegaEngine = None
    ext.PyLoadState = FakeLoadState
    sys.modules["pegaflow.pegaflow"] = ext
    ipc = types.ModuleType("pegaflow.ipc_wrapper")
    CudaIPCWrapper.__module__ = "pegaflow.ipc_wrapper"
    ipc.CudaIPCWrapper = CudaIPCWrapper
    sys.modules["pegaflow.ipc_wrapper"] = ipc
    sys.path.insert(0, str(ref_python))
    torch.cuda.synchronize = lambda *a, **k: None  # CPU-only generation


# (name, shape, dtype) — the BASELINE.json config shapes, plus layout edge cases.
CASES = [
    ("gpt2_k_separate", (256, 16, 12, 64), torch.float16),
    ("gpt2_kv_first", (2, 256, 16, 12, 64), torch.float16),
    ("llama8b_kv_first", (2, 8192, 16, 8, 128), torch.bfloat16),
    ("llama8b_blocks_first", (8192, 2, 16, 8, 128), torch.bfloat16),
    ("qwen3_8b_kv_first", (2, 2048, 16, 8, 128), torch.bfloat16),
    ("llama70b_tp8_kv_first", (2, 4096, 16, 1, 128), torch.bfloat16),
    ("llama70b_tp2_kv_first", (2, 4096, 16, 4, 128), torch.bfloat16),
    ("llama8b_fp8_kv_first", (2, 4096, 16, 8, 128), torch.uint8),
    ("fp32_scale_per_block", (4096,), torch.float32),
    ("two_blocks_ambiguous", (2, 2, 16, 8, 128), torch.bfloat16),
]


def main(argv: list[str]) -> int:
    if len(argv) < 2:
        print(__doc__.split("Usage")[1].strip(), file=sys.stderr)
        return 2
    ref_root = Path(argv[1])
    install_stubs(ref_root / "python")
    from pegaflow.connector.common import ConnectorContext, LoadIntent, PegaConnectorMetadata, SaveIntent
    from pegaflow.connector.worker import SaveTask, WorkerConnector

    # ---- registration -------------------------------------------------------
    reg_out = []
    for name, shape, dtype in CASES:
        ctx = ConnectorContext("inst", "ns", 16, 1, 1, 0, 0, FakeEngineRpcClient())
        w = WorkerConnector(ctx)
        t = torch.empty(shape, dtype=dtype, device="meta")
        _Recorder.calls = []
        w.register_kv_caches({name: t})
        (_, args), = _Recorder.calls
        (instance_id, namespace, tp_rank, tp_size, device_id, num_layers, layer_name, _wrapper,
         num_blocks, bytes_per_block, kv_stride_bytes, segments) = args
        reg_out.append({
            "case": name, "shape": list(shape), "stride": list(t.stride()), "element_size": t.element_size(),
            "num_blocks": num_blocks, "bytes_per_block": bytes_per_block, "kv_stride_bytes": kv_stride_bytes,
            "segments": segments,
        })
        w._save_queue.put(None)
        w._save_thread.join()
    (OUT / "registration.json").write_text(json.dumps(reg_out, indent=1) + "\n")

    # ---- save batching ------------------------------------------------------
    ctx = ConnectorContext("inst", "ns", 16, 3, 1, 0, 0, FakeEngineRpcClient())
    w = WorkerConnector(ctx)
    meta = PegaConnectorMetadata(save_intents={
        "reqA": SaveIntent(block_ids=(5, 9, 2), block_hashes=(b"hA0", b"hA1", b"hA2")),
        "reqB": SaveIntent(block_ids=(), block_hashes=()),
        "reqC": SaveIntent(block_ids=(7, -1), block_hashes=(b"hC0", b"hC1")),
    })
    attn = types.SimpleNamespace(block_table=object())
    no_table = types.SimpleNamespace(block_table=None)
    tasks = [
        SaveTask("layer.0", attn, meta, ["reqA", "reqB", "reqC"]),
        SaveTask("layer.1", attn, meta, ["reqA", "reqB", "reqC"]),
        SaveTask("layer.2", no_table, meta, ["reqA", "reqB", "reqC"]),
        SaveTask("layer.0", attn, meta, ["reqA"]),
    ]
    _Recorder.calls = []
    w._process_save_batch(tasks)
    saves = [a for n, a in _Recorder.calls if n == "save"]
    save_out = {
        "tasks": [{"layer": t.layer_name, "has_block_table": t.attn_metadata.block_table is not None} for t in tasks],
        "save_intents": {k: {"block_ids": list(v.block_ids), "block_hashes": [h.hex() for h in v.block_hashes]}
                         for k, v in meta.save_intents.items()},
        "rpc": [{"instance_id": a[0], "tp_rank": a[1], "device_id": a[2],
                 "saves": [[ln, list(ids), [h.hex() for h in hs]] for ln, ids, hs in a[3]]} for a in saves],
    }
    (OUT / "save_batches.json").write_text(json.dumps(save_out, indent=1) + "\n")
    w._save_queue.put(None)
    w._save_thread.join()

    # ---- load request -------------------------------------------------------
    w = WorkerConnector(ctx)
    meta = PegaConnectorMetadata(
        load_intents={
            "r1": LoadIntent(block_ids=(3, 4, 5), block_hashes=(b"a", b"b", b"c"), num_tokens=48),
            "r2": LoadIntent(block_ids=(11,), block_hashes=(b"z",), num_tokens=16),
        },
        save_intents={"r3": SaveIntent(block_ids=(1,), block_hashes=(b"q",))},
    )
    layers = {"model.layers.0.attn": types.SimpleNamespace(kv_cache=[None]),
              "model.layers.0.mlp": types.SimpleNamespace(),
              "model.layers.1.attn": types.SimpleNamespace(kv_cache=[None])}
    fwd = types.SimpleNamespace(no_compile_layers=layers)
    _Recorder.calls = []
    w.start_load_kv(meta, fwd)
    loads = [a for n, a in _Recorder.calls if n == "load"]
    load_out = {
        "load_intents": {k: {"block_ids": list(v.block_ids), "block_hashes": [h.hex() for h in v.block_hashes]}
                         for k, v in meta.load_intents.items()},
        "layers": {k: hasattr(v, "kv_cache") for k, v in layers.items()},
        "rpc": [{"instance_id": a[0], "tp_rank": a[1], "device_id": a[2], "load_state_shm": a[3],
                 "layer_names": list(a[4]), "block_ids": list(a[5]), "block_hashes": [h.hex() for h in a[6]]}
                for a in loads],
    }
    (OUT / "load_requests.json").write_text(json.dumps(load_out, indent=1) + "\n")
    w._save_queue.put(None)
    w._save_thread.join()

    # ---- request tracker traces (common.py RequestTracker) --------------------
    from pegaflow.connector.common import RequestTracker, derive_namespace

    import random

    traces = []
    for seed in range(40):
        rnd = random.Random(seed)
        nblk = rnd.randint(1, 12)
        hashes = [bytes([seed, i]) for i in range(nblk)]
        t = RequestTracker(f"r{seed}", hashes, 16, 3)
        ops, outs = [], []
        next_block = 100
        for _ in range(rnd.randint(3, 14)):
            op = rnd.choice(["lookup", "alloc", "load", "sched", "save", "layer", "finish", "hold"])
            if op == "lookup":
                args = [rnd.randint(0, nblk + 2), rnd.randint(0, nblk)]
                t.on_lookup(*args)
                out = None
            elif op == "alloc":
                k = rnd.randint(0, 4)
                args = [list(range(next_block, next_block + k)), rnd.choice([0, 0, 16, 48])]
                next_block += k
                t.on_alloc(*args)
                out = None
            elif op == "load":
                args = []
                li = t.consume_load_intent()
                out = None if li is None else [list(li.block_ids), [h.hex() for h in li.block_hashes], li.num_tokens]
            elif op == "sched":
                args = [rnd.randint(0, 40)]
                t.on_scheduled(*args)
                out = None
            elif op == "save":
                args = []
                si = t.consume_save_intent()
                out = None if si is None else [list(si.block_ids), [h.hex() for h in si.block_hashes]]
            elif op == "layer":
                args = []
                t.on_layer_saved()
                out = None
            elif op == "finish":
                args = []
                t.on_finished()
                out = None
            else:
                args = []
                out = t.should_hold_blocks()
            ops.append([op, args])
            outs.append([out, t.phase.value, t.is_done()])
        traces.append({"hashes": [h.hex() for h in hashes], "block_size": 16, "layers": 3, "ops": ops,
                       "outs": outs})
    (OUT / "tracker_traces.json").write_text(json.dumps(traces) + "\n")

    # ---- namespace derivation (common.py:283-302) -----------------------------
    cfg = types.SimpleNamespace(
        model_config=types.SimpleNamespace(model="meta-llama/Llama-3.1-8B", dtype="torch.bfloat16",
                                           get_total_num_kv_heads=lambda: 8, get_head_size=lambda: 128,
                                           get_total_num_hidden_layers=lambda: 32),
        cache_config=types.SimpleNamespace(cache_dtype="auto"))
    ns = {"factors": {"model": "meta-llama/Llama-3.1-8B", "dtype": "torch.bfloat16", "tp_size": 2,
                      "num_kv_heads": 8, "head_size": 128, "num_hidden_layers": 32, "cache_dtype": "auto"},
          "namespace": derive_namespace(cfg, 2)}
    (OUT / "namespace.json").write_text(json.dumps(ns, indent=1) + "\n")

    # ---- SGLang adapter registration (peagflow_radix_cache.py:160-250) ----------
    # configs[0] registers separate K and V tensors as segments=1 layers, as
    # the SGLang adapter does. sglang is not installed: stub the names the
    # adapter module imports (its registration code uses none of them).
    stubs = {"sglang": [], "sglang.srt": [], "sglang.srt.mem_cache": [],
             "sglang.srt.mem_cache.base_prefix_cache": ["MatchResult"],
             "sglang.srt.mem_cache.hicache_storage": ["get_hash_str"],
             "sglang.srt.mem_cache.radix_cache": ["RadixCache", "RadixKey", "TreeNode"]}
    for mod, names in stubs.items():
        m = types.ModuleType(mod)
        for n in names:
            setattr(m, n, type(n, (), {}))
        sys.modules[mod] = m
    from pegaflow.sglang.peagflow_radix_cache import PeagflowRadixCache

    sg_out = []
    for name, shape, dtype, page in [("gpt2_k_token_major", (4096, 12, 64), torch.float16, 16),
                                     ("llama8b_k_token_major", (131072, 8, 128), torch.bfloat16, 16),
                                     ("page_size_1", (256, 4, 64), torch.float16, 1),
                                     ("page_size_64", (8192, 2, 128), torch.bfloat16, 64)]:
        fake_self = types.SimpleNamespace(page_size=page, engine_client=FakeEngineRpcClient(), instance_id="inst",
                                          namespace="ns", tp_rank=0, tp_size=1, device_id=0)
        t = torch.empty(shape, dtype=dtype, device="meta")
        _Recorder.calls = []
        PeagflowRadixCache._register_single_layer(fake_self, tensor=t, layer_name=name, total_layers=24)
        (_, args), = _Recorder.calls
        sg_out.append({"case": name, "shape": list(shape), "element_size": t.element_size(), "page_size": page,
                       "num_layers": args[5], "num_blocks": args[8], "bytes_per_block": args[9],
                       "kv_stride_bytes": args[10], "segments": args[11]})
    (OUT / "sglang_registration.json").write_text(json.dumps(sg_out, indent=1) + "\n")
    print("wrote", [p.name for p in sorted(OUT.glob("*.json"))])
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
