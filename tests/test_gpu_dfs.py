"""Packed-file tier through the engine on a GPU: blocks saved from HBM are
written through to packed files whose bytes and records equal the oracle's
restatement of write_packed_file (seal_offload.rs:379-448); after pool
pressure evicts them, a query reports LOADING, the tier reads them back, and
a load restores the original bytes into new block ids."""

import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def gen(torch, shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype).cuda()


def sidecars(root: Path):
    """{file name: [(hash, BlockMeta json)] in offset order} from the sidecar files."""
    import json

    files = {}
    for meta in root.rglob("*.bin.meta"):
        rows = []
        for line in meta.read_text().splitlines()[1:]:
            parts = line.split("\t")
            if parts[0] == "block":
                rows.append((bytes.fromhex(parts[1]), parts[2]))
        rows.sort(key=lambda r: json.loads(r[1])["offset"])
        files[meta.name[:-5]] = (meta.parent, rows)
    return files


def test_write_through_evict_prefetch_restore(cuda, oracle, tmp_path):
    torch = cuda
    from pegaflow_b200 import Layout, PegaEngine, PyLoadState

    nb, n = 256, 40
    kv = [gen(torch, (2, nb, 16, 8, 128), torch.bfloat16, 10 + i) for i in range(4)]
    scale = gen(torch, (nb,), torch.float32, 99)
    names = [f"model.layers.{i}.self_attn" for i in range(4)] + ["model.layers.0.k_scale"]
    tensors = kv + [scale]
    root = tmp_path / "dfs"
    eng = PegaEngine(16 << 20, enable_lfu_admission=False, dfs_root=str(root))
    try:
        for nm, t in zip(names, tensors):
            lay = Layout.from_tensor(t)
            eng.register_context_layer("inst", "ns", 0, nm, lay.data_ptr, lay.size_bytes, lay.num_blocks,
                                       lay.bytes_per_block, lay.kv_stride_bytes, lay.segments, 0, 1, len(names))
        rng = np.random.default_rng(0)
        src = rng.permutation(nb)[:n].tolist()
        ha = [f"reqA-{i}".encode() for i in range(n)]
        eng.batch_save_kv_blocks("inst", 0, 0, [(nm, src, ha) for nm in names])
        assert eng.dfs_flush(30)
        assert eng.dfs_stats()["written_blocks"] == n

        # Files and records against the oracle: slot l of block i is
        # (K, V) of layer l for the KV layers, the 4-byte scale otherwise.
        def slots_of(h):
            b = src[ha.index(h)]
            out = [(t[0, b].contiguous().view(torch.uint8).cpu().numpy().tobytes(),
                    t[1, b].contiguous().view(torch.uint8).cpu().numpy().tobytes()) for t in kv]
            out.append((scale[b:b + 1].view(torch.uint8).cpu().numpy().tobytes(), None))
            return out

        seen = 0
        for fname, (d, rows) in sidecars(root).items():
            data, metas = oracle.dfs_pack([slots_of(h) for h, _ in rows], fname)
            assert (d / fname).read_bytes() == data, fname
            assert [m for _, m in rows] == metas, fname
            seen += len(rows)
        assert seen == n

        # Pool pressure: a second request evicts the first from the pool.
        hb = [f"reqB-{i}".encode() for i in range(n)]
        eng.batch_save_kv_blocks("inst", 0, 0, [(nm, src, hb) for nm in names])
        # B's write-through holds its blocks until written; a read-back that
        # needs their pool memory before then fails and is simply retried on
        # the next query (as in the reference). Let it finish first.
        assert eng.dfs_flush(30)
        assert eng.count_prefix_hit_blocks("inst", ha) == 0
        q = eng.query_prefetch("inst", ha)
        assert q["prefetch_state"] == "loading" and q["loading_blocks"] == n
        assert eng.dfs_flush(30)
        q = eng.query_prefetch("inst", ha)
        assert q == {"hit_blocks": n, "prefetch_state": "ready", "loading_blocks": 0, "missing_blocks": 0}, (
            q, eng.dfs_stats())

        # Restore request A from the blocks read back, into new ids.
        dst = rng.permutation(nb)[:n].tolist()
        before = [t.clone() for t in tensors]
        s = PyLoadState()
        eng.batch_load_kv_blocks("inst", 0, 0, s.shm_name(), names, dst, ha)
        t0 = time.time()
        while not s.is_ready():
            assert time.time() - t0 < 60
            time.sleep(0.001)
        assert s.get_state() == 1
        torch.cuda.synchronize()
        src_t, dst_t = torch.tensor(src, device="cuda"), torch.tensor(dst, device="cuda")
        for t, b in zip(kv, before[:4]):
            assert torch.equal(t.index_select(1, dst_t), b.index_select(1, src_t))
        assert torch.equal(scale.index_select(0, dst_t), before[4].index_select(0, src_t))
    finally:
        eng.close()
