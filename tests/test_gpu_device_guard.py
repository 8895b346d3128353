"""The library leaves the caller's current device (its CUDA context) as it
found it.

Every entry point that works on a given device makes that device current for
the call and then puts the caller's context back. Without that, an inference
engine thread working on device 1 that saves blocks of device 0 would find
device 0 current afterwards, and its next torch or CUDA call would run on the
wrong GPU. The one-GPU test checks the case of a thread that had no context at
all (it must still have none); the two-GPU test checks a save, a load, a peer
copy and an engine save for device 0 issued while device 1 is current.
"""

import ctypes
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def current_context() -> int | None:
    cu = ctypes.CDLL("libcuda.so.1")
    ctx = ctypes.c_void_p()
    assert cu.cuCtxGetCurrent(ctypes.byref(ctx)) == 0
    return ctx.value


def kv(torch, shape, seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(torch.bfloat16).to(device)


def round_trip_specs(t, src, dst, pool_ptr):
    from pegaflow_b200 import Layout, LoadSpec, SaveSpec

    lay = Layout.from_tensor(t)
    n, unit = len(src), lay.bytes_per_block
    ks = np.arange(n, dtype=np.uint64) * unit + pool_ptr
    return SaveSpec(lay, src, pool_ptr, pool_ptr + n * unit), LoadSpec(lay, dst, ks, ks + n * unit)


def test_thread_without_context_still_has_none(cuda, native):
    torch = cuda
    from pegaflow_b200 import Executor, PinnedBuffer

    t = kv(torch, (2, 64, 16, 8, 128), 1, "cuda:0")
    src, dst = np.arange(0, 16), np.arange(32, 48)
    pool = PinnedBuffer(2 * 16 * 32768)
    save, load = round_trip_specs(t, src, dst, pool.ptr)
    ex = Executor(0)
    seen = {}

    def worker():
        seen["before"] = current_context()
        ex.save([save])
        ex.load([load])
        native.check(native.lib.pf_save_blocks_noalloc(0, None, 0, None))
        seen["after"] = current_context()

    th = threading.Thread(target=worker)
    th.start()
    th.join()
    assert seen["before"] is None
    assert seen["after"] is None
    assert torch.equal(t[:, 32:48], t[:, 0:16])


def test_calls_for_device_0_leave_device_1_current(cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from pegaflow_b200 import Executor, Layout, P2PSpec, PegaEngine, PinnedBuffer

    t0 = kv(torch, (2, 64, 16, 8, 128), 2, "cuda:0")
    t1 = kv(torch, (2, 64, 16, 8, 128), 3, "cuda:1")
    pool = PinnedBuffer(2 * 16 * 32768)
    save, load = round_trip_specs(t0, np.arange(0, 16), np.arange(32, 48), pool.ptr)
    ex0 = Executor(0)
    torch.cuda.set_device(1)
    try:
        ctx1 = current_context()
        ex0.save([save])
        assert torch.cuda.current_device() == 1 and current_context() == ctx1
        ex0.load([load])
        assert torch.cuda.current_device() == 1 and current_context() == ctx1
        # Pull GPU0 -> GPU1 issued by device 0's executor as a push.
        ex0.p2p([P2PSpec(Layout.from_tensor(t0), Layout.from_tensor(t1), np.arange(8), np.arange(8))], 1, push=True)
        assert torch.cuda.current_device() == 1 and current_context() == ctx1
        e = PegaEngine(64 << 20, enable_lfu_admission=False)
        lay = Layout.from_tensor(t0)
        e.register_context_layer("g", "ns", 0, "l0", lay.data_ptr, lay.size_bytes, lay.num_blocks,
                                 lay.bytes_per_block, lay.kv_stride_bytes, lay.segments, 0, 1, 1)
        e.batch_save_kv_blocks("g", 0, 0, [("l0", list(range(8)), [f"h{i}".encode() for i in range(8)])])
        assert torch.cuda.current_device() == 1 and current_context() == ctx1
        e.close()
        torch.cuda.synchronize(0)
        assert torch.equal(t0[:, 32:48], t0[:, 0:16])
        assert torch.equal(t1[:, 0:8], t0[:, 0:8].to("cuda:1"))
    finally:
        torch.cuda.set_device(0)
