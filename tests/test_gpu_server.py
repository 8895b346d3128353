"""Two processes on one GPU, as deployed: the engine server
(`python -m pegaflow_b200.server`) maps this test process's KV tensors over
CUDA IPC; the test drives it with EngineRpcClient and checks the restored
bytes and the per-layer completion words."""

import pickle
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture
def server(cuda, engine_server):
    client, _ = engine_server()
    return client


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
