import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def native():
    """The native library, built in-tree if needed (nvcc; no GPU required)."""
    from pegaflow_b200 import build as b

    b.build()
    from pegaflow_b200 import _native

    return _native


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    return o


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch


@pytest.fixture
def engine_server():
    """Starts `python -m pegaflow_b200.server` as its own process (CUDA IPC
    cannot map a handle into the process that made it) and returns
    (connected EngineRpcClient, endpoint); extra command-line flags may be
    passed. The server is shut down at teardown."""
    import socket
    import subprocess
    import time

    started = []

    def start(*extra: str):
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        proc = subprocess.Popen([sys.executable, "-m", "pegaflow_b200.server", "--addr", f"127.0.0.1:{port}",
                                 "--pool-size", "512mb", "--disable-lfu-admission", "--log-level", "warning", *extra],
                                cwd=str(ROOT), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                env=dict(os.environ, PYTHONPATH=str(ROOT)))
        from pegaflow_b200 import EngineRpcClient

        endpoint = f"http://127.0.0.1:{port}"
        client, deadline = None, time.time() + 120
        while client is None:
            try:
                client = EngineRpcClient(endpoint, connect_timeout_s=1.0)
            except RuntimeError:
                if proc.poll() is not None or time.time() > deadline:
                    out = proc.stdout.read().decode(errors="replace") if proc.stdout else ""
                    proc.kill()
                    pytest.fail(f"server did not start: {out[-2000:]}")
        started.append((proc, client))
        return client, endpoint

    yield start
    for proc, client in started:
        try:
            client.shutdown()
        except RuntimeError:
            pass
        try:
            proc.wait(timeout=30)
        except subprocess.TimeoutExpired:
            proc.kill()
            proc.wait()
