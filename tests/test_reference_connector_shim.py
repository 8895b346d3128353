"""The reference's own Python package, unmodified, running on this library.

The stand-in for the compiled ``pegaflow.pegaflow`` extension
(pegaflow_b200/compat/pegaflow.py) is installed into a temporary copy of the
reference's ``pegaflow`` package made of links to its files. The test then
imports the package the way vLLM does, checks that its engine classes are
this library's, and drives the reference's scheduler-side connector
(connector/scheduler.py, unmodified) against this library's gRPC server: a
request whose prefix lies in a packed file is answered "retry later" while
the server prefetches it, then with the prefix's tokens once the blocks are in
the pool (scheduler.py:36-80, 221-262).

CPU only (a plain-memory engine; vLLM's connector base imports without a
GPU). Skipped when the reference tree is not beside this repository or named
by PEGAFLOW_REFERENCE_TREE.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def reference_package() -> Path | None:
    cands = [os.environ.get("PEGAFLOW_REFERENCE_TREE"), str(ROOT.parent / "reference")]
    for c in cands:
        if c and (Path(c) / "python" / "pegaflow" / "connector" / "scheduler.py").exists():
            return Path(c) / "python" / "pegaflow"
    return None


SCRIPT = r'''
import json, os, sys, time, types
import numpy as np

import pegaflow
from pegaflow.pegaflow import EngineRpcClient, PegaEngine, PyLoadState
from pegaflow_b200.client import EngineRpcClient as OurClient
from pegaflow_b200.engine import PegaEngine as OurEngine, PyLoadState as OurLoadState

assert (EngineRpcClient, PegaEngine, PyLoadState) == (OurClient, OurEngine, OurLoadState)
assert (pegaflow.EngineRpcClient, pegaflow.PegaEngine, pegaflow.PyLoadState) == (OurClient, OurEngine, OurLoadState)
assert pegaflow.__file__.startswith(sys.argv[2])
from pegaflow.connector import KVConnectorRole, PegaKVConnector  # the reference connector (imports vLLM)
from pegaflow.connector.common import ConnectorContext
from pegaflow.connector.scheduler import SchedulerConnector

from oracle import oracle
from pegaflow_b200.server import TensorRegistry, serve

# One packed file in namespace "ns": four blocks of one split slot each.
dfs = sys.argv[1]
hashes = [b"blk%d" % i for i in range(4)]
data, metas = oracle.dfs_pack([[(bytes([i]) * 4096, bytes([100 + i]) * 4096)] for i in range(4)], "f0.bin")
os.makedirs(os.path.join(dfs, "ns"))
with open(os.path.join(dfs, "ns", "f0.bin"), "wb") as f:
    f.write(data)
side = ["pegaflow-packed-file 1", "member\tns:f0", "timestamp_ms\t1", f"size\t{len(data)}",
        "file_meta\t" + oracle.dfs_file_meta(hashes, len(data))]
side += [f"block\t{h.hex()}\t{m}" for h, m in zip(hashes, metas)]
with open(os.path.join(dfs, "ns", "f0.bin.meta"), "w") as f:
    f.write("\n".join(side) + "\n")

engine = OurEngine(1 << 20, pool_kind="host", dfs_root=dfs)
fake = np.zeros(2 * 16 * 4096, np.uint8)
server, _, port = serve(engine, "127.0.0.1:0", TensorRegistry(lambda d, w: (fake, fake.ctypes.data, fake.nbytes, d)))
client = EngineRpcClient(f"http://127.0.0.1:{port}", connect_timeout_s=5)
try:
    assert client.register_context("inst", "ns", 0, 1, 0, 1, "L0", b"w", 16, 4096, 16 * 4096, 2) == (True, "")
    ctx = ConnectorContext(instance_id="inst", namespace="ns", block_size=16, num_layers=1, tp_size=1,
                           tp_rank=None, device_id=None, engine_client=client)
    sched = SchedulerConnector(ctx)
    miss = sched.get_num_new_matched_tokens(types.SimpleNamespace(request_id="M", num_tokens=48,
                                                                  block_hashes=[b"x", b"y", b"z"]), 0)
    req = types.SimpleNamespace(request_id="A", num_tokens=80, block_hashes=hashes + [b"new"])
    answers, deadline = [], time.time() + 60
    while True:
        answers.append(sched.get_num_new_matched_tokens(req, 0))
        if answers[-1][0] is not None:
            break
        assert time.time() < deadline, "prefetch did not finish"
        time.sleep(0.01)
    print(json.dumps({"miss": miss, "first": answers[0], "last": answers[-1], "queries": len(answers),
                      "connector": PegaKVConnector.__module__}))
finally:
    client.close()
    server.stop(0)
    engine.close()
'''


def test_reference_scheduler_connector_runs_on_this_library(native, tmp_path):
    ref = reference_package()
    if ref is None:
        pytest.skip("the reference tree is not available")
    from pegaflow_b200.compat import install

    pkg = tmp_path / "site" / "pegaflow"
    pkg.mkdir(parents=True)
    for entry in ref.iterdir():
        if entry.name == "__pycache__" or entry.name.startswith("pegaflow.") and entry.suffix == ".so":
            continue
        (pkg / entry.name).symlink_to(entry)
    shim = install(pkg)
    assert shim.read_text() == (ROOT / "pegaflow_b200" / "compat" / "pegaflow.py").read_text()
    dfs = tmp_path / "dfs"
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(tmp_path / "site"), str(ROOT)]))
    p = subprocess.run([sys.executable, "-c", SCRIPT, str(dfs), str(pkg)], capture_output=True, text=True,
                       timeout=600, cwd=str(tmp_path), env=env)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    out = json.loads(p.stdout.strip().splitlines()[-1])
    assert out["connector"] == "pegaflow.connector"
    assert out["miss"] == [0, False]
    # While the server reads the packed file into the pool, the reference
    # scheduler is told to retry; then it gets the 4 cached blocks (64 tokens).
    assert out["first"] == [None, False]
    assert out["last"] == [64, True]
