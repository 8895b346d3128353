"""Tensor-parallel sharding on 2+ GPUs through one engine (as one reference
server serves all TP ranks of a node): each rank registers its own KV head
shard on its own device, saves concurrently into the shared pinned pool, and
a block becomes visible only when every rank's slots are filled
(slot = layer * tp_size + tp_rank, pegaflow-core/src/lib.rs:205-219;
seal gate storage.rs:161-193). Skipped on single-GPU machines."""

import threading
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def kv(torch, shape, seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(torch.bfloat16).to(device)


def host_bytes(t):
    import torch

    return t.detach().cpu().contiguous().view(-1).view(torch.uint8).numpy().copy()


def test_tp2_shards_seal_only_when_every_rank_saved(cuda, oracle):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from pegaflow_b200 import Layout, PegaEngine, PyLoadState
    from pegaflow_b200.ranks import tp_heads

    tp, layers, nb = 2, 3, 256
    e = PegaEngine(512 << 20, enable_lfu_admission=False)
    m = oracle.EngineModel()
    tensors = {}
    for r in range(tp):
        lo, hi = tp_heads(8, r, tp)
        for li in range(layers):
            t = kv(torch, (2, nb, 16, hi - lo, 128), 10 * r + li, f"cuda:{r}")
            tensors[(r, li)] = t
            lay = Layout.from_tensor(t)
            name = f"model.layers.{li}.attn"
            e.register_context_layer("tp", "ns", r, name, lay.data_ptr, lay.size_bytes, lay.num_blocks,
                                     lay.bytes_per_block, lay.kv_stride_bytes, 2, r, tp, layers)
            ol = oracle.Layout(lay.size_bytes, lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, 2)
            m.register_context_layer("tp", "ns", r, name, host_bytes(t), ol, r, tp, layers)
    names = [f"model.layers.{li}.attn" for li in range(layers)]
    ids = np.random.default_rng(0).permutation(nb)[:100].tolist()
    hs = [b"blk%d" % i for i in range(100)]

    e.batch_save_kv_blocks("tp", 0, 0, [(n, ids, hs) for n in names])
    m.batch_save("tp", 0, 0, [(n, ids, hs) for n in names])
    assert e.count_prefix_hit_blocks("tp", hs) == 0  # rank 1's slots are missing

    # Both ranks save concurrently (rank 0's entries are already inflight: skipped).
    errs = []

    def save(rank):
        try:
            e.batch_save_kv_blocks("tp", rank, rank, [(n, ids, hs) for n in names])
        except Exception as ex:  # pragma: no cover - reported below
            errs.append(ex)

    th = [threading.Thread(target=save, args=(r,)) for r in range(tp)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert not errs
    m.batch_save("tp", 1, 1, [(n, ids, hs) for n in names])
    assert e.count_prefix_hit_blocks("tp", hs) == 100 == m.count_prefix_hit_blocks("tp", hs)

    dst = np.random.default_rng(1).permutation(nb)[:100].tolist()
    for r in range(tp):
        s = PyLoadState()
        e.batch_load_kv_blocks("tp", r, r, s.shm_name(), names, dst, hs)
        t0 = time.time()
        while not s.is_ready():
            assert time.time() - t0 < 60
            time.sleep(0.001)
        assert s.get_state() == 1
        assert m.batch_load("tp", r, r, names, dst, hs)[0] == 1
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    for r in range(tp):
        for li, n in enumerate(names):
            _, gpu = m.instances["tp"].regs[(r, n)]
            np.testing.assert_array_equal(host_bytes(tensors[(r, li)]), gpu)


def test_pool_is_pinned_for_every_device(cuda):
    """The pool is allocated Portable|Mapped, so a copy engine on any device
    moves it at pinned speed and zero-copy kernels on any device can read it."""
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer, SaveSpec

    pool = PinnedBuffer(64 * 65536)
    src = kv(torch, (2, 128, 16, 8, 128), 1, "cuda:0")
    Executor(0).save([SaveSpec(Layout.from_tensor(src), np.arange(64), pool.ptr, pool.ptr + 64 * 32768)])
    dst = torch.zeros((2, 128, 16, 8, 128), dtype=torch.bfloat16, device="cuda:1")
    ks = np.array([pool.ptr + i * 32768 for i in range(64)], np.uint64)
    Executor(1, load_mode="direct").load([LoadSpec(Layout.from_tensor(dst), np.arange(64) + 10, ks, ks + 64 * 32768)])
    torch.cuda.synchronize(1)
    assert torch.equal(dst[:, 10:74].cpu(), src[:, :64].cpu())


def test_device_pools_keep_each_gpus_blocks(cuda):
    """numa_pools="device": one pool per GPU. Filling GPU 1's pool evicts
    GPU 1's oldest blocks and never GPU 0's, which a single shared pool of
    the same total size would evict first (they are the least recently
    used). Bytes restored from either pool are the saved ones."""
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from pegaflow_b200 import Layout, PegaEngine, PyLoadState

    block = 16 * 8 * 128 * 2  # one K or V segment of a [2, nb, 16, 8, 128] bf16 layer
    per_dev = 64 * 2 * block  # room for 64 blocks of one layer per GPU

    def run(mode):
        e = PegaEngine(2 * per_dev, enable_lfu_admission=False, numa_pools=mode)
        ts = {}
        for d in (0, 1):
            t = kv(torch, (2, 256, 16, 8, 128), 40 + d, f"cuda:{d}")
            lay = Layout.from_tensor(t)
            e.register_context_layer(f"i{d}", f"ns{d}", d, "L0", lay.data_ptr, lay.size_bytes, lay.num_blocks,
                                     lay.bytes_per_block, lay.kv_stride_bytes, lay.segments, 0, 1, 1)
            ts[d] = t
        old = [f"d0-{i}".encode() for i in range(32)]
        e.batch_save_kv_blocks("i0", 0, 0, [("L0", list(range(32)), old)])
        for k in range(6):  # 6 x 32 blocks on GPU 1: more than its pool holds
            hs = [f"d1-{k}-{i}".encode() for i in range(32)]
            e.batch_save_kv_blocks("i1", 0, 1, [("L0", list(range(32)), hs)])
        hit0 = e.count_prefix_hit_blocks("i0", old)
        if mode == "device":  # restore GPU 0's blocks elsewhere and compare
            s = PyLoadState()
            e.batch_load_kv_blocks("i0", 0, 0, s.shm_name(), ["L0"], list(range(100, 132)), old)
            deadline = time.time() + 60
            while not s.is_ready():
                assert time.time() < deadline
            assert s.get_state() == 1
            torch.cuda.synchronize(0)
            assert torch.equal(ts[0][:, 100:132], ts[0][:, 0:32])
        m = e.metrics()
        e.close()
        return hit0, m["cache_block_evictions"]

    hit_dev, ev_dev = run("device")
    hit_one, ev_one = run("off")
    assert hit_dev == 32 and ev_dev > 0  # GPU 1 evicted its own blocks only
    assert hit_one == 0 and ev_one > 0   # one pool: GPU 0's older blocks went first
