"""Two processes on one GPU, as deployed: the engine server
(`python -m pegaflow_b200.server`) maps this test process's KV tensors over
CUDA IPC; the test drives it with EngineRpcClient and checks the restored
bytes and the per-layer completion words."""

import os
import pickle
import socket
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def server(cuda):
    port = _port()
    proc = subprocess.Popen([sys.executable, "-m", "pegaflow_b200.server", "--addr", f"127.0.0.1:{port}",
                             "--pool-size", "512mb", "--disable-lfu-admission", "--log-level", "warning"],
                            cwd=str(ROOT), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                            env=dict(os.environ, PYTHONPATH=str(ROOT)))
    from pegaflow_b200 import EngineRpcClient

    client = None
    deadline = time.time() + 120
    while client is None:
        try:
            client = EngineRpcClient(f"http://127.0.0.1:{port}", connect_timeout_s=1.0)
        except RuntimeError:
            if proc.poll() is not None or time.time() > deadline:
                out = proc.stdout.read().decode(errors="replace") if proc.stdout else ""
                pytest.fail(f"server did not start: {out[-2000:]}")
    yield client
    try:
        client.shutdown()
    except RuntimeError:
        pass
    try:
        proc.wait(timeout=30)
    except subprocess.TimeoutExpired:
        proc.kill()
        proc.wait()


def test_register_save_query_load_over_ipc(server, cuda):
    torch = cuda
    from pegaflow_b200 import CudaIPCWrapper, Layout, PyLoadState

    client = server
    g = torch.Generator().manual_seed(0)
    layers = {f"model.layers.{i}.self_attn": torch.randn((2, 128, 16, 8, 128), generator=g).to(torch.bfloat16).cuda()
              for i in range(4)}
    for name, t in layers.items():
        lay = Layout.from_tensor(t)
        ok, msg = client.register_context("inst", "ns", 0, 1, 0, len(layers), name, pickle.dumps(CudaIPCWrapper(t)),
                                          lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, lay.segments)
        assert ok, msg
    src = np.random.default_rng(0).permutation(128)[:40].tolist()
    hashes = [b"h%03d" % i for i in range(40)]
    before = {n: t[:, src].clone() for n, t in layers.items()}
    torch.cuda.synchronize()
    assert client.save("inst", 0, 0, [(n, src, hashes) for n in layers]) == (True, "")
    assert client.query("inst", hashes)["hit_blocks"] == 40
    for t in layers.values():
        t.zero_()
    torch.cuda.synchronize()
    dst = np.random.default_rng(1).permutation(128)[:40].tolist()
    s = PyLoadState(len(layers))
    assert client.load("inst", 0, 0, s.shm_name(), list(layers), dst, hashes) == (True, "")
    for i in range(len(layers)):
        assert s.wait_layer(i, timeout_s=60)
    t0 = time.time()
    while not s.is_ready():
        assert time.time() - t0 < 60
        time.sleep(0.001)
    assert s.get_state() == 1
    torch.cuda.synchronize()
    for n, t in layers.items():
        assert torch.equal(t[:, dst], before[n]), n
    assert client.unregister_context("inst") == (True, "")
