"""GPU end-to-end parity of PegaEngine (register -> save -> query -> load)
against the oracle's EngineModel restatement of pegaflow-core/src/lib.rs."""

import json
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def kv(torch, shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype).cuda()


def host_bytes(t):
    import torch

    return t.detach().cpu().contiguous().view(-1).view(torch.uint8).numpy().copy()


def wait_state(s, timeout=60.0):
    t0 = time.time()
    while not s.is_ready():
        if time.time() - t0 > timeout:
            raise TimeoutError("load did not complete")
        time.sleep(0.001)
    return s.get_state()


class Pair:
    """The engine and the model driven with the same calls."""

    def __init__(self, torch, oracle, pool=1 << 30, **kw):
        from pegaflow_b200 import PegaEngine

        self.torch = torch
        self.oracle = oracle
        self.e = PegaEngine(pool, enable_lfu_admission=False, **kw)
        self.m = oracle.EngineModel()
        self.tensors = {}

    def register(self, name, t, inst="inst", ns="ns", tp_rank=0, tp_size=1, num_layers=1):
        from pegaflow_b200 import Layout

        lay = Layout.from_tensor(t)
        self.tensors[name] = t
        self.e.register_context_layer(inst, ns, 0, name, lay.data_ptr, lay.size_bytes, lay.num_blocks,
                                      lay.bytes_per_block, lay.kv_stride_bytes, lay.segments, tp_rank, tp_size,
                                      num_layers)
        ol = self.oracle.Layout(lay.size_bytes, lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes,
                                lay.segments)
        self.m.register_context_layer(inst, ns, 0, name, host_bytes(t), ol, tp_rank, tp_size, num_layers)

    def save(self, saves, inst="inst", tp_rank=0):
        self.e.batch_save_kv_blocks(inst, tp_rank, 0, saves)
        self.m.batch_save(inst, tp_rank, 0, saves)

    def load(self, layers, ids, hashes, inst="inst", tp_rank=0):
        from pegaflow_b200 import PyLoadState

        s = PyLoadState()
        try:
            self.e.batch_load_kv_blocks(inst, tp_rank, 0, s.shm_name(), layers, ids, hashes)
            err = None
        except RuntimeError as ex:
            err = str(ex)
        state = wait_state(s)
        mstate, merr = self.m.batch_load(inst, tp_rank, 0, layers, ids, hashes)
        assert state == mstate, (err, merr)
        if merr is not None and err is not None:
            assert err == str(merr)
        return state

    def check_caches(self):
        self.torch.cuda.synchronize()
        for name, t in self.tensors.items():
            _, gpu = self.m.instances["inst"].regs[(0, name)]
            np.testing.assert_array_equal(host_bytes(t), gpu, err_msg=name)

    def check_slots(self, hashes, slots, ns="ns"):
        """Pool bytes of every sealed (hash, slot) equal the model's payload."""
        import ctypes

        for h in hashes:
            for slot in slots:
                p = self.m.slot_payload(ns, h, slot)
                assert p is not None
                k, v, size = self.e.slot_info(ns, h, slot)
                kb = np.ctypeslib.as_array((ctypes.c_uint8 * p.k.size).from_address(k))
                np.testing.assert_array_equal(kb, p.k)
                if p.v is not None:
                    vb = np.ctypeslib.as_array((ctypes.c_uint8 * p.v.size).from_address(v))
                    np.testing.assert_array_equal(vb, p.v)


def hashes_for(prefix, n):
    return [f"{prefix}-{i}".encode() for i in range(n)]


def test_gpt2_config_through_engine(cuda, oracle):
    """BASELINE config 0 through the engine API: 24 segments=1 layers
    (separate K and V of 12 layers), 64 blocks saved, restored elsewhere."""
    torch = cuda
    p = Pair(torch, oracle, pool=256 << 20)
    names = [f"L{i // 2}_{'kv'[i % 2]}" for i in range(24)]
    for i, n in enumerate(names):
        p.register(n, kv(torch, (256, 16, 12, 64), torch.float16, 100 + i), num_layers=24)
    src = torch.randperm(256, generator=torch.Generator().manual_seed(1))[:64].tolist()
    rest = sorted(set(range(256)) - set(src))
    dst = [rest[i] for i in torch.randperm(len(rest), generator=torch.Generator().manual_seed(2))[:64].tolist()]
    hs = hashes_for("gpt2", 64)
    p.save([(n, src, hs) for n in names])
    assert p.e.count_prefix_hit_blocks("inst", hs) == 64 == p.m.count_prefix_hit_blocks("inst", hs)
    p.check_slots(hs, range(24))
    assert p.load(names, dst, hs) == 1
    p.check_caches()


def test_kv_first_layers_seal_and_dedup(cuda, oracle):
    torch = cuda
    p = Pair(torch, oracle)
    names = [f"model.layers.{i}.self_attn" for i in range(4)]
    for i, n in enumerate(names):
        p.register(n, kv(torch, (2, 512, 16, 8, 128), torch.bfloat16, 10 + i), num_layers=4)
    ids = np.random.default_rng(0).permutation(512)[:300].tolist()
    hs = hashes_for("req", 300)
    # Only three of four layers: nothing is sealed yet (storage.rs:161-193).
    p.save([(n, ids, hs) for n in names[:3]])
    assert p.e.count_prefix_hit_blocks("inst", hs) == 0
    assert p.e.metrics()["inflight_blocks"] == 300
    used_before = p.e.pool_usage()[0]
    p.save([(n, ids, hs) for n in names[:3]])  # already inflight for those slots: skipped
    assert p.e.pool_usage()[0] == used_before
    p.save([(names[3], ids, hs)])
    assert p.e.count_prefix_hit_blocks("inst", hs) == 300
    p.check_slots(hs[:20], range(4))
    # A prefix stops at the first miss.
    assert p.e.count_prefix_hit_blocks("inst", hs[:10] + [b"missing"] + hs[10:]) == 10
    dst = np.random.default_rng(1).permutation(512)[:300].tolist()
    assert p.load(names, dst, hs) == 1
    p.check_caches()


def test_save_batch_golden_replay(cuda, oracle):
    """Replay the save RPC the reference's connector builds (duplicated layer
    entry, negative ids) and compare pool bytes with the model."""
    torch = cuda
    g = json.loads((GOLDEN / "save_batches.json").read_text())
    (rpc,) = g["rpc"]
    p = Pair(torch, oracle)
    for i, n in enumerate(["layer.0", "layer.1", "layer.2"]):
        p.register(n, kv(torch, (2, 16, 16, 2, 64), torch.bfloat16, i), num_layers=3)
    saves = [(ln, ids, [bytes.fromhex(h) for h in hs]) for ln, ids, hs in rpc["saves"]]
    p.save(saves)
    p.save([("layer.2", [5, 9, 2, 7], [bytes.fromhex(h) for h in ["684130", "684131", "684132", "684330"]])])
    hs = [bytes.fromhex(h) for h in ["684130", "684131", "684132", "684330"]]
    assert p.e.count_prefix_hit_blocks("inst", hs) == 4
    p.check_slots(hs, range(3))
    assert p.load(["layer.0", "layer.1", "layer.2"], [1, 3, -1, 4], hs) == 1
    p.check_caches()


def test_layer_wise_completion_words(cuda, oracle):
    """A LoadState with the per-layer extension gets each layer's word raised
    by the kernels as that layer lands (before the batch state turns 1);
    layers with no blocks are raised at once."""
    torch = cuda
    from pegaflow_b200 import PyLoadState

    p = Pair(torch, oracle)
    names = [f"L{i}" for i in range(6)]
    for i, n in enumerate(names):
        p.register(n, kv(torch, (2, 256, 16, 8, 128), torch.bfloat16, 30 + i), num_layers=6)
    ids = list(range(0, 200))
    hs = hashes_for("lw", 200)
    p.save([(n, ids, hs) for n in names])
    s = PyLoadState(len(names))
    dst = list(range(40, 240))
    p.e.batch_load_kv_blocks("inst", 0, 0, s.shm_name(), names, dst, hs)
    for li in range(len(names)):
        assert s.wait_layer(li, timeout_s=60), li
    assert wait_state(s) == 1
    assert all(s.layer_ready(i) for i in range(len(names)))
    # The load's phase timings: the first layer is ready within the task's
    # time from queueing to completion.
    p.e.wait_loads(0, 30.0)
    m = p.e.metrics()
    assert m["load_calls"] == 1 and m["load_transfer_ms"] > 0
    assert 0 < m["load_first_layer_ms"] <= m["load_queue_ms"] + m["load_setup_ms"] + m["load_transfer_ms"] + 1e-3
    assert m["load_lookup_ms"] >= 0 and m["load_ms"] >= m["load_transfer_ms"]
    p.m.batch_load("inst", 0, 0, names, dst, hs)
    p.check_caches()


def test_load_errors_match_model(cuda, oracle):
    torch = cuda
    p = Pair(torch, oracle)
    p.register("a", kv(torch, (2, 32, 16, 8, 128), torch.bfloat16, 1), num_layers=1)
    hs = hashes_for("x", 4)
    p.save([("a", [0, 1, 2, 3], hs)])
    assert p.load(["a"], [0, 1], [b"nope", hs[0]]) == -1          # missing hash
    assert p.load(["zz"], [0, 1], hs[:2]) == -1                    # unknown layer
    assert p.load(["a"], [0, 1], hs[:2], tp_rank=1) == -1          # tp_rank out of range
    assert p.load(["a"], [0, 32], hs[:2]) == -1                    # destination past the registration
    assert p.load(["a"], [5, 6, 7], hs[:2]) == 1                    # zip: extra ids are ignored
    assert p.e.metrics()["load_failures"] >= 1
    p.check_caches()


def test_lru_eviction_makes_room(cuda, oracle):
    """Pool exhaustion reclaims least-recently-used sealed blocks (storage.rs:405-433)."""
    torch = cuda
    from pegaflow_b200 import PegaEngine, Layout

    t = kv(torch, (2, 64, 16, 8, 128), torch.bfloat16, 3)
    lay = Layout.from_tensor(t)
    e = PegaEngine(40 * 65536 + 4096, enable_lfu_admission=False)
    e.register_context_layer("i", "ns", 0, "L", lay.data_ptr, lay.size_bytes, lay.num_blocks, lay.bytes_per_block,
                             lay.kv_stride_bytes, lay.segments, 0, 1, 1)
    a, b = hashes_for("a", 16), hashes_for("b", 16)
    e.save_kv_blocks("i", 0, 0, "L", list(range(16)), a)
    assert e.count_prefix_hit_blocks("i", a) == 16
    e.save_kv_blocks("i", 0, 0, "L", list(range(16, 32)), b)
    e.save_kv_blocks("i", 0, 0, "L", list(range(32, 48)), hashes_for("c", 16))
    assert e.count_prefix_hit_blocks("i", a) == 0  # evicted first
    assert e.count_prefix_hit_blocks("i", hashes_for("c", 16)) == 16
    assert e.metrics()["cache_block_evictions"] >= 16
    with pytest.raises(RuntimeError, match="pinned pool exhausted"):
        e.save_kv_blocks("i", 0, 0, "L", list(range(64)), hashes_for("big", 64))


def test_save_while_a_load_runs(cuda, oracle):
    """A save issued while a queued load is still moving (the save on the
    calling thread, the load on the device's load thread, on separate lanes)
    gives the same pool and cache bytes as the two run one after the other.
    The load's destination blocks and the save's source blocks are disjoint."""
    torch = cuda
    from pegaflow_b200 import PyLoadState

    p = Pair(torch, oracle)
    names = [f"model.layers.{i}.self_attn" for i in range(4)]
    for i, n in enumerate(names):
        p.register(n, kv(torch, (2, 1024, 16, 8, 128), torch.bfloat16, 50 + i), num_layers=4)
    perm = np.random.default_rng(7).permutation(1024)
    a_src, load_dst, b_src = perm[:300].tolist(), perm[300:600].tolist(), perm[600:900].tolist()
    ha, hb = hashes_for("dup-a", 300), hashes_for("dup-b", 300)
    p.save([(n, a_src, ha) for n in names])
    s = PyLoadState(len(names))
    p.e.batch_load_kv_blocks("inst", 0, 0, s.shm_name(), names, load_dst, ha)
    p.e.batch_save_kv_blocks("inst", 0, 0, [(n, b_src, hb) for n in names])
    assert wait_state(s) == 1
    assert p.m.batch_load("inst", 0, 0, names, load_dst, ha) == (1, None)
    p.m.batch_save("inst", 0, 0, [(n, b_src, hb) for n in names])
    assert p.e.count_prefix_hit_blocks("inst", hb) == 300
    p.check_slots(hb[:50] + hb[-50:], range(4))
    p.check_caches()


def test_concurrent_saves_of_two_instances(cuda, oracle):
    """Two instances on one device saving from two threads at once (each save
    call orders on a stream of its own; the device's save lane runs them in
    turn): every sealed block holds its own source bytes."""
    import threading

    torch = cuda
    p = Pair(torch, oracle)
    insts = {"i1": ("ns1", 60), "i2": ("ns2", 70)}
    for inst, (ns, seed) in insts.items():
        for j in range(2):
            p.register(f"{inst}.L{j}", kv(torch, (2, 512, 16, 8, 128), torch.bfloat16, seed + j), inst=inst, ns=ns,
                       num_layers=2)
    work = {inst: [(np.random.default_rng(seed + k).permutation(512)[:40].tolist(), hashes_for(f"{inst}-{k}", 40))
                   for k in range(6)] for inst, (_, seed) in insts.items()}
    errors = []

    def run(inst):
        try:
            for ids, hs in work[inst]:
                p.e.batch_save_kv_blocks(inst, 0, 0, [(f"{inst}.L{j}", ids, hs) for j in range(2)])
        except Exception as e:  # reported by the main thread
            errors.append(e)

    threads = [threading.Thread(target=run, args=(inst,)) for inst in work]
    for t in threads:
        t.start()
    for t in threads:
        t.join(120)
    assert not errors and not any(t.is_alive() for t in threads)
    for inst, (ns, _) in insts.items():
        for ids, hs in work[inst]:
            p.m.batch_save(inst, 0, 0, [(f"{inst}.L{j}", ids, hs) for j in range(2)])
            assert p.e.count_prefix_hit_blocks(inst, hs) == 40
            p.check_slots(hs[:4] + hs[-4:], range(2), ns=ns)
