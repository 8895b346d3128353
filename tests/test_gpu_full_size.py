"""Parity at BASELINE.json's full sizes, by properties that need no CPU
oracle (the same code paths are checked byte for byte against the oracle at
small sizes in test_gpu_transfer.py and test_gpu_engine.py):

  * pool layout: each layer's K region equals K[src_ids] and its V region
    V[src_ids], compared on the GPU with a torch gather of the source;
  * round trip: after the load, block dst_ids[i] of every layer equals the
    source's block src_ids[i], and every other block is unchanged;
  * block ids include the first and the last block of the cache.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def gen(torch, shape, dtype, seed):
    """Seeded values generated on the GPU (the CPU path is too slow at 16 GiB)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    if dtype == torch.uint8:
        return torch.randint(0, 256, shape, generator=g, device="cuda", dtype=torch.uint8)
    return torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).to(dtype)


def ids_with_ends(nb, n, seed, exclude=None):
    """n distinct ids in seeded order, containing 0 and nb-1 (unless excluded)."""
    rng = np.random.default_rng(seed)
    pool = np.arange(nb) if exclude is None else np.setdiff1d(np.arange(nb), exclude)
    ids = rng.permutation(pool)[:n]
    for end in (0, nb - 1):
        if end in pool and end not in ids:
            ids[rng.integers(n)] = end
    assert len(set(ids.tolist())) == n
    return ids


def as_bytes(t):
    return t.contiguous().view(-1).view(__import__("torch").uint8)


@pytest.mark.parametrize("order", ["sorted", "shuffled"])
def test_llama8b_config_full_size_executor(cuda, order):
    """32 layers of [2, 8192, 16, 8, 128] bf16 (16 GiB), 640 blocks."""
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer, SaveSpec

    nb, n, layers = 8192, 640, 32
    caches = [gen(torch, (2, nb, 16, 8, 128), torch.bfloat16, 1000 + i) for i in range(layers)]
    if order == "sorted":
        src, dst = np.arange(n), np.arange(n) + 4096
        src[-1] = nb - 1
    else:
        src = ids_with_ends(nb, n, 3)
        dst = ids_with_ends(nb, n, 4, exclude=src)
    seg = 16 * 8 * 128 * 2
    pool = PinnedBuffer(layers * n * 2 * seg)
    ex = Executor(0)
    saves, loads = [], []
    for i, t in enumerate(caches):
        lay = Layout.from_tensor(t)
        k = pool.ptr + i * 2 * n * seg
        v = k + n * seg
        saves.append(SaveSpec(lay, src, k, v))
        loads.append(LoadSpec(lay, dst, np.arange(n, dtype=np.uint64) * seg + k,
                              np.arange(n, dtype=np.uint64) * seg + v))
    ex.save(saves)
    torch.cuda.synchronize()
    host = torch.from_numpy(pool.numpy())
    src_t = torch.from_numpy(src).cuda()
    for i, t in enumerate(caches):
        region = host[i * 2 * n * seg:(i + 1) * 2 * n * seg].cuda()
        expect = torch.cat([as_bytes(t[0].index_select(0, src_t)), as_bytes(t[1].index_select(0, src_t))])
        assert torch.equal(region, expect), f"pool layout of layer {i}"
    before = [t.clone() for t in caches]
    ex.load(loads)
    torch.cuda.synchronize()
    dst_t = torch.from_numpy(dst).cuda()
    untouched = torch.from_numpy(np.setdiff1d(np.arange(nb), dst)).cuda()
    for i, (t, b) in enumerate(zip(caches, before)):
        assert torch.equal(t.index_select(1, dst_t), b.index_select(1, src_t)), f"restored blocks of layer {i}"
        assert torch.equal(t.index_select(1, untouched), b.index_select(1, untouched)), f"other blocks of layer {i}"


def _engine_round_trip(torch, names, caches, axes, src, dst, pool_bytes):
    """Register every layer of one instance, save src with one hash list for
    all layers, load into dst with per-layer words, check on the GPU.
    axes[i] is the block axis of caches[i]."""
    import time

    from pegaflow_b200 import Layout, PegaEngine, PyLoadState

    eng = PegaEngine(pool_bytes, enable_lfu_admission=False)
    try:
        for nm, t in zip(names, caches):
            lay = Layout.from_tensor(t)
            eng.register_context_layer("full", "ns", 0, nm, lay.data_ptr, lay.size_bytes, lay.num_blocks,
                                       lay.bytes_per_block, lay.kv_stride_bytes, lay.segments, 0, 1, len(names))
        hashes = [f"full-{i}".encode() for i in range(len(src))]
        src_l, dst_l = src.tolist(), dst.tolist()
        eng.batch_save_kv_blocks("full", 0, 0, [(nm, src_l, hashes) for nm in names])
        assert eng.count_prefix_hit_blocks("full", hashes) == len(src)
        before = [t.clone() for t in caches]
        s = PyLoadState(len(names))
        eng.batch_load_kv_blocks("full", 0, 0, s.shm_name(), names, dst_l, hashes)
        deadline = time.time() + 120
        while not s.is_ready():
            assert time.time() < deadline, "load did not complete"
            time.sleep(0.001)
        assert s.get_state() == 1
        assert all(s.layer_ready(i) for i in range(len(names)))
        s.close()
        torch.cuda.synchronize()
        src_t, dst_t = torch.from_numpy(src).cuda(), torch.from_numpy(dst).cuda()
        for nm, t, b, ax in zip(names, caches, before, axes):
            untouched = torch.from_numpy(np.setdiff1d(np.arange(t.shape[ax]), dst)).cuda()
            assert torch.equal(t.index_select(ax, dst_t), b.index_select(ax, src_t)), nm
            assert torch.equal(t.index_select(ax, untouched), b.index_select(ax, untouched)), nm
    finally:
        eng.close()


def test_llama70b_tp8_shard_full_size_engine(cuda):
    """configs[3] at TP8, one rank's shard through the engine: 80 layers of
    [2, 4096, 16, 1, 128] bf16 (4 KiB segments), 2,048 blocks."""
    torch = cuda
    nb, n = 4096, 2048
    names = [f"model.layers.{i}.self_attn" for i in range(80)]
    caches = [gen(torch, (2, nb, 16, 1, 128), torch.bfloat16, 2000 + i) for i in range(80)]
    src = ids_with_ends(nb, n, 5)
    dst = ids_with_ends(nb, n, 6)  # may overlap src: the pool holds the saved bytes
    _engine_round_trip(torch, names, caches, [1] * 80, src, dst, 80 * n * 8192 + (64 << 20))


def test_fp8_with_scales_full_request_engine(cuda):
    """configs[4]'s layout: 32 fp8 KV layers [2, NB, 16, 8, 128] plus 32 fp32
    per-block scale layers [NB] (4-byte blocks), one 16K-token request
    (1,024 blocks), restored into other ids."""
    torch = cuda
    nb, n = 4096, 1024
    names, caches = [], []
    for i in range(32):
        names.append(f"model.layers.{i}.self_attn")
        caches.append(gen(torch, (2, nb, 16, 8, 128), torch.uint8, 3000 + i))
    for i in range(32):
        names.append(f"model.layers.{i}.k_scale")
        caches.append(gen(torch, (nb,), torch.float32, 4000 + i))
    src = ids_with_ends(nb, n, 7)
    dst = ids_with_ends(nb, n, 8, exclude=src)
    # One instance of 64 layers: a block seals once its 32 KV and 32 scale
    # slots are all in (blocks sit on axis 1 of a KV layer, axis 0 of a scale).
    _engine_round_trip(torch, names, caches, [1] * 32 + [0] * 32, src, dst,
                       32 * n * (2 * 16384 + 4) + (64 << 20))
