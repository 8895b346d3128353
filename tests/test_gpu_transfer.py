"""GPU parity of the transfer executor against the CPU oracle (bit-exact).

Every test moves seeded KV bytes HBM -> pinned pool -> HBM through the sm_100a
kernels (staged ring + copy engine, and zero-copy direct mode) and compares
pool bytes and restored cache bytes with the oracle's restatement of the
reference copies (oracle/pf_oracle.c, oracle/oracle.py).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MODES = ["staged", "direct"]


def kv(torch, shape, dtype, seed):
    """Seeded ~N(0,1) values generated on the CPU, then moved to the GPU."""
    g = torch.Generator().manual_seed(seed)
    if dtype in (torch.uint8,):
        t = torch.randint(0, 256, shape, generator=g, dtype=torch.uint8)
    else:
        t = torch.randn(shape, generator=g, dtype=torch.float32).to(dtype)
    return t.cuda()


def host_bytes(t):
    return t.detach().cpu().contiguous().view(-1).view(__import__("torch").uint8).numpy().copy()


def olayout(oracle, lay):
    return oracle.Layout(lay.size_bytes, lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, lay.segments)


def save_and_check(cuda, oracle, ex, layers_and_ids, pool):
    """Save every (tensor, ids) into consecutive pool regions; check pool bytes
    against the oracle. Returns per-layer (k_ptr, v_ptr, layout)."""
    from pegaflow_b200 import Layout, SaveSpec

    specs, regions, expect = [], [], []
    off = 0
    for t, ids in layers_and_ids:
        lay = Layout.from_tensor(t)
        n = len(ids)
        if lay.split:
            k, v = pool.ptr + off, pool.ptr + off + n * lay.bytes_per_block
            off += 2 * n * lay.bytes_per_block
        else:
            k, v = pool.ptr + off, None
            off += n * lay.block_size_bytes
        off = (off + 255) // 256 * 256
        specs.append(SaveSpec(lay, np.asarray(ids), k, v))
        regions.append((k, v, lay))
        kr, vr = oracle.np_save_layer(olayout(oracle, lay), host_bytes(t), ids)
        expect.append((kr, vr))
    ex.save(specs)
    view = pool.numpy()
    for (k, v, lay), (kr, vr) in zip(regions, expect):
        got_k = view[k - pool.ptr:k - pool.ptr + kr.size]
        np.testing.assert_array_equal(got_k, kr)
        if vr is not None:
            got_v = view[v - pool.ptr:v - pool.ptr + vr.size]
            np.testing.assert_array_equal(got_v, vr)
    return regions


def load_and_check(cuda, oracle, ex, dst_tensors, regions, dst_ids, layer_flags=False):
    """Load every region into `dst_ids` and compare with the oracle. With
    `layer_flags`, the load also raises per-layer flags (which start its chunk
    schedule small) and every flag must be up afterwards."""
    from pegaflow_b200 import LoadSpec, PinnedBuffer

    specs, expect = [], []
    for t, (k, v, lay), ids in zip(dst_tensors, regions, dst_ids):
        from pegaflow_b200 import Layout

        dlay = Layout.from_tensor(t)
        n = len(ids)
        unit = lay.bytes_per_block if lay.split else lay.block_size_bytes
        ks = np.array([k + i * unit for i in range(n)], dtype=np.uint64)
        vs = np.array([v + i * unit for i in range(n)], dtype=np.uint64) if lay.split else None
        specs.append(LoadSpec(dlay, np.asarray(ids), ks, vs))
        ref = host_bytes(t)
        oracle.load_layer(olayout(oracle, dlay), ref, ids, [int(x) for x in ks],
                          [int(x) for x in vs] if vs is not None else None)
        expect.append(ref)
    if layer_flags:
        flags = PinnedBuffer(8 * len(specs))
        flags.numpy()[:] = 0
        ex.load(specs, layer_done=flags.ptr)
    else:
        ex.load(specs)
    cuda.cuda.synchronize()
    for t, ref in zip(dst_tensors, expect):
        np.testing.assert_array_equal(host_bytes(t), ref)
    if layer_flags:
        assert flags.numpy(np.int64).tolist() == [1] * len(specs)


@pytest.mark.parametrize("mode", MODES)
def test_gpt2_config_round_trip(cuda, oracle, mode):
    """12 layers of separate K and V tensors [256,16,12,64]
    fp16 (registered as segments=1 layers, like the SGLang adapter), 64 source
    blocks by seeded permutation, restored into 64 other seeded ids."""
    torch = cuda
    from pegaflow_b200 import Executor, PinnedBuffer

    ex = Executor(0, save_mode=mode, load_mode=mode)
    tensors = [kv(torch, (256, 16, 12, 64), torch.float16, seed=100 + i) for i in range(24)]
    src = torch.randperm(256, generator=torch.Generator().manual_seed(1))[:64].numpy()
    rest = np.setdiff1d(np.arange(256), src)
    dst = rest[torch.randperm(rest.size, generator=torch.Generator().manual_seed(2))[:64].numpy()]
    pool = PinnedBuffer(24 * 64 * 24576 + 24 * 256)
    regions = save_and_check(torch, oracle, ex, [(t, src) for t in tensors], pool)
    before = [host_bytes(t) for t in tensors]
    load_and_check(torch, oracle, ex, tensors, regions, [dst] * 24)
    # Byte-exact: every destination block now equals its source block; others untouched.
    bpb = 24576
    for t, b in zip(tensors, before):
        after = host_bytes(t).reshape(256, bpb)
        bb = b.reshape(256, bpb)
        np.testing.assert_array_equal(after[dst], bb[src])
        untouched = np.setdiff1d(np.arange(256), dst)
        np.testing.assert_array_equal(after[untouched], bb[untouched])


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("order", ["sorted", "shuffled"])
def test_llama_kv_first_layers(cuda, oracle, mode, order):
    """Config 1 shape (KV-first [2, NB, 16, 8, 128] bf16) with 640 blocks,
    sorted-contiguous and seeded-shuffled ids, on a reduced block count."""
    torch = cuda
    from pegaflow_b200 import Executor, PinnedBuffer

    nb = 1024
    ex = Executor(0, save_mode=mode, load_mode=mode)
    src_t = [kv(torch, (2, nb, 16, 8, 128), torch.bfloat16, seed=7 + i) for i in range(3)]
    if order == "sorted":
        src, dst = np.arange(640), np.arange(640) + 200
    else:
        src = torch.randperm(nb, generator=torch.Generator().manual_seed(3))[:640].numpy()
        dst = torch.randperm(nb, generator=torch.Generator().manual_seed(4))[:640].numpy()
    pool = PinnedBuffer(3 * 640 * 65536 + 4096)
    regions = save_and_check(torch, oracle, ex, [(t, src) for t in src_t], pool)
    dst_t = [kv(torch, (2, nb, 16, 8, 128), torch.bfloat16, seed=70 + i) for i in range(3)]
    load_and_check(torch, oracle, ex, dst_t, regions, [dst] * 3)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("chunk,first", [(64 << 10, 0), (200 << 10, 0), (16 << 20, 0), (1 << 20, 8 << 10),
                                         (300 << 10, 9 << 10)])
def test_many_chunks_and_mixed_layouts(cuda, oracle, mode, chunk, first):
    """Small staging chunks split units across chunks and slots wrap many
    times; layers mix split, blocks-first, 4-byte scales and unaligned units.
    A small first chunk makes every chunk of the growth schedule differ in
    size (8 KiB, 16 KiB, ... up to the slot): loads with per-layer flags
    start there; saves and flagless loads start at half a slot."""
    torch = cuda
    from pegaflow_b200 import Executor, PinnedBuffer

    ex = Executor(0, save_mode=mode, load_mode=mode, staging_chunk_bytes=chunk, staging_slots=2,
                  first_chunk_bytes=first)
    layers = [
        kv(torch, (2, 64, 16, 2, 128), torch.bfloat16, 1),   # split, 8 KiB units
        kv(torch, (64, 16, 4, 64), torch.float16, 2),         # blocks-first, 8 KiB
        kv(torch, (64,), torch.float32, 3),                   # fp32 per-block scale: 4-byte units
        kv(torch, (64, 3, 4), torch.uint8, 4),                # 12-byte blocks: unaligned
        kv(torch, (2, 64, 5, 9), torch.uint8, 5),             # split, 45-byte units
        kv(torch, (2, 64, 16, 8, 128), torch.uint8, 6),       # fp8-like, 16 KiB units
    ]
    rng = np.random.default_rng(11)
    ids = [rng.permutation(64)[:40] for _ in layers]
    pool = PinnedBuffer(8 << 20)
    regions = save_and_check(torch, oracle, ex, list(zip(layers, ids)), pool)
    dst = [rng.permutation(64)[:40] for _ in layers]
    load_and_check(torch, oracle, ex, layers, regions, dst)
    dst = [rng.permutation(64)[:40] for _ in layers]
    load_and_check(torch, oracle, ex, layers, regions, dst, layer_flags=True)


@pytest.mark.parametrize("mode", MODES)
def test_first_and_last_blocks_of_the_cache(cuda, oracle, mode):
    """Block ids 0 and num_blocks-1 on both sides, so the last block's bytes
    end exactly at the end of the registered tensor (split, blocks-first and
    4-byte scale layouts)."""
    torch = cuda
    from pegaflow_b200 import Executor, PinnedBuffer

    ex = Executor(0, save_mode=mode, load_mode=mode)
    layers = [kv(torch, (2, 64, 16, 8, 128), torch.bfloat16, 1), kv(torch, (64, 2, 16, 4, 64), torch.float16, 2),
              kv(torch, (64,), torch.float32, 3)]
    src, dst = np.array([63, 0, 5, 62]), np.array([0, 63, 1, 62])
    pool = PinnedBuffer(1 << 20)
    regions = save_and_check(torch, oracle, ex, [(t, src) for t in layers], pool)
    load_and_check(torch, oracle, ex, layers, regions, [dst] * 3)


def test_empty_and_single_block_layers(cuda, oracle):
    torch = cuda
    from pegaflow_b200 import Executor, PinnedBuffer

    ex = Executor(0)
    layers = [kv(torch, (2, 8, 16, 128), torch.bfloat16, 1), kv(torch, (2, 8, 16, 128), torch.bfloat16, 2),
              kv(torch, (8, 256), torch.float16, 3)]
    ids = [np.array([], dtype=np.int64), np.array([7]), np.array([0])]
    pool = PinnedBuffer(1 << 20)
    regions = save_and_check(torch, oracle, ex, list(zip(layers, ids)), pool)
    load_and_check(torch, oracle, ex, layers, regions, [np.array([], dtype=np.int64), np.array([3]), np.array([5])])


@pytest.mark.parametrize("mode", MODES)
def test_repeated_destinations_keep_the_last_block(cuda, oracle, mode):
    """The reference copies a layer's blocks in list order, so a destination
    listed twice ends up with the later block; the kernels keep that."""
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer

    t = kv(torch, (2, 16, 16, 8, 128), torch.bfloat16, 1)
    lay = Layout.from_tensor(t)
    pool = PinnedBuffer(8 * 65536)
    pool.numpy()[:] = np.random.default_rng(0).integers(0, 256, pool.nbytes, dtype=np.uint8)
    ids = np.array([3, 5, 3, 9, 5, 3])
    ks = np.array([pool.ptr + i * 32768 for i in range(6)], np.uint64)
    vs = ks + 6 * 32768
    ref = host_bytes(t)
    oracle.load_layer(olayout(oracle, lay), ref, ids, [int(x) for x in ks], [int(x) for x in vs])
    Executor(0, load_mode=mode).load([LoadSpec(lay, ids, ks, vs)])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bytes(t), ref)


@pytest.mark.parametrize("mode", MODES)
def test_self_overlapping_layouts_load_in_list_order(cuda, oracle, mode):
    """Layouts whose blocks share bytes (K/V interleaved with stride ==
    bytes_per_block, or 3 strided segments) take the ordered copy path and end
    byte-identical to the reference's sequential copies."""
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer

    raw = kv(torch, (40 * 4096,), torch.uint8, 2)
    layouts = [Layout(raw.data_ptr(), 33 * 4096, 32, 4096, 4096, 2),      # contiguous, 8 KiB blocks overlap
               Layout(raw.data_ptr(), 40 * 4096, 8, 4096, 9 * 4096, 3)]   # 3 strided segments
    rng = np.random.default_rng(7)
    for lay in layouts:
        pool = PinnedBuffer(40 * lay.block_size_bytes)
        pool.numpy()[:] = rng.integers(0, 256, pool.nbytes, dtype=np.uint8)
        nb_ok = [b for b in range(lay.num_blocks) if b * lay.bytes_per_block + lay.block_size_bytes <= lay.size_bytes]
        ids = rng.choice(nb_ok, size=12)
        ks = np.array([pool.ptr + i * lay.block_size_bytes for i in range(12)], np.uint64)
        ref = host_bytes(raw)
        ol = oracle.Layout(lay.size_bytes, lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, lay.segments)
        oracle.load_layer(ol, ref, ids, [int(x) for x in ks], None)
        Executor(0, load_mode=mode).load([LoadSpec(lay, ids, ks, None)])
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host_bytes(raw), ref)


def test_out_of_range_ids_fail_before_any_copy(cuda):
    torch = cuda
    from pegaflow_b200 import Executor, Layout, PinnedBuffer, SaveSpec

    ex = Executor(0)
    t = kv(torch, (2, 16, 16, 128), torch.bfloat16, 1)
    pool = PinnedBuffer(1 << 20)
    pool.numpy()[:] = 7
    with pytest.raises(RuntimeError, match="block 16 out of range"):
        ex.save([SaveSpec(Layout.from_tensor(t), np.array([0, 16]), pool.ptr, pool.ptr + 4096 * 2)])
    with pytest.raises(RuntimeError, match="block -1 out of range"):
        ex.save([SaveSpec(Layout.from_tensor(t), np.array([-1]), pool.ptr, pool.ptr + 4096)])
    # The first bad id in list order is the one reported, not the largest.
    with pytest.raises(RuntimeError, match="block 17 out of range"):
        ex.save([SaveSpec(Layout.from_tensor(t), np.array([3, 17, 5, 40]), pool.ptr, pool.ptr + 4096 * 4)])
    assert (pool.numpy() == 7).all()


def test_load_past_the_registration_names_the_first_bad_block(cuda):
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer

    ex = Executor(0)
    t = kv(torch, (32, 16, 128), torch.bfloat16, 2)  # blocks-first, 4 KiB blocks
    before = host_bytes(t)
    pool = PinnedBuffer(1 << 20)
    ks = np.array([pool.ptr + i * 4096 for i in range(4)], np.uint64)
    with pytest.raises(RuntimeError, match="Block 35 segment 0 exceeds registered memory"):
        ex.load([LoadSpec(Layout.from_tensor(t), np.array([2, 35, 3, 40]), ks, None)])
    with pytest.raises(RuntimeError, match="negative block index -2"):
        ex.load([LoadSpec(Layout.from_tensor(t), np.array([2, -2, 3, 40]), ks, None)])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bytes(t), before)  # nothing was copied


def test_direct_mode_refuses_unregistered_host_memory(cuda):
    torch = cuda
    from pegaflow_b200 import Executor, Layout, SaveSpec

    ex = Executor(0, save_mode="direct")
    t = kv(torch, (2, 16, 16, 128), torch.bfloat16, 1)
    buf = np.zeros(1 << 20, np.uint8)
    with pytest.raises(RuntimeError, match="pinned memory allocated by this library"):
        ex.save([SaveSpec(Layout.from_tensor(t), np.array([1]), buf.ctypes.data, buf.ctypes.data + 8192)])


def test_kv_tensor_must_be_device_memory(cuda):
    from pegaflow_b200 import Executor, Layout, PinnedBuffer, SaveSpec

    ex = Executor(0)
    host = np.zeros(2 * 16 * 4096, np.uint8)
    lay = Layout(host.ctypes.data, host.nbytes, 16, 4096, 16 * 4096, 2)
    pool = PinnedBuffer(1 << 20)
    with pytest.raises(RuntimeError, match="not (CUDA|device) memory"):
        ex.save([SaveSpec(lay, np.array([1]), pool.ptr, pool.ptr + 4096)])


def test_reference_copy_strategy_produces_the_same_bytes(cuda, oracle):
    """The restated reference copy path (per-segment D2H, merged H2D runs)
    and the kernels agree byte for byte."""
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer, SaveSpec, refcopy_load, refcopy_save

    t = kv(torch, (2, 128, 16, 8, 128), torch.bfloat16, 9)
    lay = Layout.from_tensor(t)
    ids = np.random.default_rng(5).permutation(128)[:50]
    a, b = PinnedBuffer(50 * 65536), PinnedBuffer(50 * 65536)
    Executor(0).save([SaveSpec(lay, ids, a.ptr, a.ptr + 50 * 32768)])
    refcopy_save(0, [SaveSpec(lay, ids, b.ptr, b.ptr + 50 * 32768)])
    np.testing.assert_array_equal(a.numpy(), b.numpy())
    d1 = kv(torch, (2, 128, 16, 8, 128), torch.bfloat16, 10)
    d2 = d1.clone()
    dst = np.random.default_rng(6).permutation(128)[:50]
    ks = np.array([a.ptr + i * 32768 for i in range(50)], np.uint64)
    vs = ks + 50 * 32768
    Executor(0).load([LoadSpec(Layout.from_tensor(d1), dst, ks, vs)])
    runs = refcopy_load(0, [LoadSpec(Layout.from_tensor(d2), dst, ks, vs)])
    torch.cuda.synchronize()
    assert torch.equal(d1, d2)
    assert runs >= 2


def test_layer_done_flags(cuda):
    """Per-layer completion words are raised for every layer of a load."""
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer

    layers = [kv(torch, (2, 32, 16, 8, 128), torch.bfloat16, i) for i in range(5)]
    pool = PinnedBuffer(5 * 10 * 65536)
    flags = PinnedBuffer(5 * 8)
    flags.numpy()[:] = 0
    specs = []
    for li, t in enumerate(layers):
        base = pool.ptr + li * 10 * 65536
        ks = np.array([base + i * 32768 for i in range(10)], np.uint64)
        ids = np.arange(10) if li != 3 else np.array([], dtype=np.int64)
        specs.append(LoadSpec(Layout.from_tensor(t), ids, ks[: len(ids)], (ks + 10 * 32768)[: len(ids)]))
    ex = Executor(0, staging_chunk_bytes=256 << 10, staging_slots=2)
    stream = torch.cuda.Stream()
    ex.load(specs, stream=stream.cuda_stream, layer_done=flags.ptr)
    stream.synchronize()
    assert flags.numpy(np.int64).tolist() == [1, 1, 1, 1, 1]


def test_stream_ordered_save_and_stats(cuda):
    torch = cuda
    from pegaflow_b200 import Executor, Layout, PinnedBuffer, SaveSpec

    t = kv(torch, (2, 256, 16, 8, 128), torch.bfloat16, 1)
    pool = PinnedBuffer(200 * 65536)
    ex = Executor(0)
    ex.set_timing(True)
    ex.reset_stats()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        t.add_(1)  # ordered before the save on the same stream
    ex.save([SaveSpec(Layout.from_tensor(t), np.arange(200), pool.ptr, pool.ptr + 200 * 32768)], stream=s.cuda_stream)
    s.synchronize()
    st = ex.stats()
    assert st["kernel_launches"] >= 1 and st["timed_launches"] == st["kernel_launches"]
    assert st["kernel_ms"] > 0 and st["bytes_saved"] == 200 * 65536
    ref = t[0, :200].contiguous().view(torch.uint8).cpu().numpy().reshape(-1)
    np.testing.assert_array_equal(pool.numpy()[: ref.size], ref)


@pytest.mark.parametrize("mode", MODES)
def test_save_and_load_run_at_once_on_two_streams(cuda, oracle, mode):
    """A save and a load issued back to back on two caller streams go to the
    executor's two lanes and overlap. They touch disjoint blocks of one KV
    cache; each moves exactly its own bytes, over several staging chunks per
    lane. A second save, ordered after the load by an event on the caller
    side, sees the restored blocks."""
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer, SaveSpec

    bpb, n = 32768, 96
    cache = kv(torch, (2, 256, 16, 8, 128), torch.bfloat16, 11)
    lay = Layout.from_tensor(cache)
    perm = torch.randperm(256, generator=torch.Generator().manual_seed(13)).numpy()
    save_ids, load_ids = perm[:n], perm[n:2 * n]
    pool = PinnedBuffer(3 * 2 * n * bpb)
    view = pool.numpy()
    # Region 1 receives the save; region 2 holds seeded blocks to restore.
    region2 = pool.ptr + 2 * n * bpb
    blocks = np.random.default_rng(14).integers(0, 256, 2 * n * bpb, dtype=np.uint8)
    view[2 * n * bpb:4 * n * bpb] = blocks
    ks = np.array([region2 + i * bpb for i in range(n)], np.uint64)
    vs = ks + n * bpb
    want_save = oracle.np_save_layer(olayout(oracle, lay), host_bytes(cache), save_ids)
    want_load = host_bytes(cache)
    oracle.load_layer(olayout(oracle, lay), want_load, load_ids, [int(x) for x in ks], [int(x) for x in vs])

    ex = Executor(0, save_mode=mode, load_mode=mode, staging_chunk_bytes=1 << 20, staging_slots=2,
                  first_chunk_bytes=256 << 10)
    s_save, s_load = torch.cuda.Stream(), torch.cuda.Stream()
    ex.save([SaveSpec(lay, save_ids, pool.ptr, pool.ptr + n * bpb)], stream=s_save.cuda_stream)
    ex.load([LoadSpec(lay, load_ids, ks, vs)], stream=s_load.cuda_stream)
    loaded = torch.cuda.Event()
    loaded.record(s_load)
    s_save.wait_event(loaded)
    region3 = pool.ptr + 4 * n * bpb
    ex.save([SaveSpec(lay, load_ids, region3, region3 + n * bpb)], stream=s_save.cuda_stream)
    torch.cuda.synchronize()

    np.testing.assert_array_equal(view[:n * bpb], want_save[0])
    np.testing.assert_array_equal(view[n * bpb:2 * n * bpb], want_save[1])
    np.testing.assert_array_equal(host_bytes(cache), want_load)
    np.testing.assert_array_equal(view[4 * n * bpb:6 * n * bpb], blocks)


def test_saves_and_loads_from_two_threads(cuda, oracle):
    """One executor driven by a saving thread and a loading thread at once
    (each lane serialises its own calls; the counters are shared): every
    transfer moves its own bytes, and the counters add up."""
    import threading

    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer, SaveSpec

    bpb, n, reps = 32768, 64, 12
    cache = kv(torch, (2, 512, 16, 8, 128), torch.bfloat16, 21)
    lay = Layout.from_tensor(cache)
    perm = np.random.default_rng(22).permutation(512)
    save_ids, load_ids = perm[:n], perm[n:2 * n]
    pool = PinnedBuffer(2 * 2 * n * bpb)
    view = pool.numpy()
    src = pool.ptr + 2 * n * bpb
    blocks = np.random.default_rng(23).integers(0, 256, 2 * n * bpb, dtype=np.uint8)
    view[2 * n * bpb:] = blocks
    ks = np.array([src + i * bpb for i in range(n)], np.uint64)
    want_save = oracle.np_save_layer(olayout(oracle, lay), host_bytes(cache), save_ids)
    want_load = host_bytes(cache)
    oracle.load_layer(olayout(oracle, lay), want_load, load_ids, [int(x) for x in ks], [int(x) for x in ks + n * bpb])

    ex = Executor(0, staging_chunk_bytes=1 << 20, staging_slots=2, first_chunk_bytes=128 << 10)
    ex.set_timing(True)
    ex.reset_stats()
    errors = []

    def run(fn):
        try:
            stream = torch.cuda.Stream()
            for _ in range(reps):
                fn(stream)
            stream.synchronize()
        except Exception as e:  # reported by the main thread
            errors.append(e)

    save = lambda s: ex.save([SaveSpec(lay, save_ids, pool.ptr, pool.ptr + n * bpb)], stream=s.cuda_stream)
    load = lambda s: ex.load([LoadSpec(lay, load_ids, ks, ks + n * bpb)], stream=s.cuda_stream)
    threads = [threading.Thread(target=run, args=(save,)), threading.Thread(target=run, args=(load,))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(120)
    assert not errors and not any(t.is_alive() for t in threads)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(view[:n * bpb], want_save[0])
    np.testing.assert_array_equal(view[n * bpb:2 * n * bpb], want_save[1])
    np.testing.assert_array_equal(host_bytes(cache), want_load)
    st = ex.stats()
    assert st["bytes_saved"] == st["bytes_loaded"] == reps * 2 * n * bpb
    assert st["timed_launches"] == st["kernel_launches"] > 2 * reps
    assert st["kernel_bytes"] == 2 * 2 * reps * 2 * n * bpb
