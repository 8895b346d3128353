"""The N>1 path on CPU: two gloo ranks run the process-per-GPU plumbing
(shards, seeds, cross-rank timing reduction) and move their own KV head shard
through the CPU oracle. No GPU; no collective touches the data."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from pegaflow_b200.ranks import block_lists, pool_region, tp_heads


def test_shard_arithmetic():
    assert [tp_heads(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        tp_heads(8, 0, 3)
    regions = [pool_region(10 << 30, r, 8) for r in range(8)]
    for (o1, s1), (o2, _) in zip(regions, regions[1:]):
        assert o1 + s1 <= o2
    s0, d0 = block_lists(4096, 2048, 0, "shuffled")
    s1, _ = block_lists(4096, 2048, 1, "shuffled")
    assert len(set(s0)) == 2048 and not np.array_equal(s0, s1)
    # Sources and destinations are disjoint, in both orders, so a restore never
    # overwrites a source block.
    for order in ("shuffled", "sorted"):
        for nb, n in ((4096, 2048), (8192, 640), (256, 64)):
            s, d = block_lists(nb, n, 0, order)
            assert len(set(s)) == n and len(set(d)) == n and not set(s) & set(d)
            assert max(s.max(), d.max()) < nb


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from oracle import oracle
    from pegaflow_b200.ranks import Ranks

    r = Ranks.from_env("gloo", timeout_s=60)
    try:
        # Each rank owns 8/world heads of a [2, NB, 16, 8, 128]-shaped layer.
        lo, hi = tp_heads(8, r.rank, r.world)
        nb, bs, hd = 64, 16, 128
        seg = bs * (hi - lo) * hd * 2
        L = oracle.Layout(2 * nb * seg, nb, seg, nb * seg, 2)
        gpu = np.random.default_rng(100 + r.rank).integers(0, 256, L.size_bytes, dtype=np.uint8)
        src, dst = block_lists(nb, 16, r.rank, "shuffled")
        k = np.zeros(16 * seg, np.uint8)
        v = np.zeros(16 * seg, np.uint8)
        oracle.save_layer(L, gpu, src, k, v)
        restored = np.zeros_like(gpu)
        oracle.load_layer(L, restored, dst, [k.ctypes.data + i * seg for i in range(16)],
                          [v.ctypes.data + i * seg for i in range(16)])
        ok = all(np.array_equal(restored[d * seg:(d + 1) * seg], gpu[s * seg:(s + 1) * seg]) for s, d in zip(src, dst))
        r.barrier()
        slowest = r.max(float(r.rank + 1))
        fastest = r.min(float(r.rank + 1))
        total = r.sum(float(seg))
        assert r.gather(float(10 * r.rank + 1)) == [float(10 * i + 1) for i in range(r.world)]
        # The bench's byte check: verified only when every rank verified.
        assert r.all_true(ok) is ok
        assert r.all_true(r.rank == 0) is False
        r.host_barrier()
        out.put((r.rank, ok, slowest, fastest, total, (lo, hi)))
    finally:
        r.close()


def test_two_gloo_ranks_save_and_restore_their_own_shards(oracle):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [res[1] for res in results] == [True, True]
    assert all(res[2] == 2.0 and res[3] == 1.0 for res in results)  # max/min over ranks
    assert results[0][5] == (0, 4) and results[1][5] == (4, 8)       # disjoint head shards
    seg = 16 * 4 * 128 * 2
    assert all(res[4] == 2 * seg for res in results)
