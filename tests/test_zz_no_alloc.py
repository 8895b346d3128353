"""pf_save_blocks_noalloc: the save path for callers that cannot allocate.

Some callers cannot call cudaMalloc while they save, for example an inference
engine whose caching allocator or KV pool already owns all free HBM. The
no-allocation entry point keeps its scratch in fixed device arrays inside the
library. These tests call it through the C ABI and check that it writes
exactly the pool bytes the regular executor save writes, on two calls in a
row (the second call finds the first call's leftovers in the shared scratch),
and that a save too large for the fixed scratch is refused.

The file sorts last so a run that stops at the first failure has already run
every other test.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def kv(torch, shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    if dtype == torch.uint8:
        return torch.randint(0, 256, shape, generator=g, dtype=torch.uint8).cuda()
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype).cuda()


def specs_for(tensors, ids_list, pool_ptr):
    from pegaflow_b200 import Layout, SaveSpec

    specs, off = [], 0
    for t, ids in zip(tensors, ids_list):
        lay = Layout.from_tensor(t)
        n = len(ids)
        if lay.split:
            specs.append(SaveSpec(lay, np.asarray(ids), pool_ptr + off, pool_ptr + off + n * lay.bytes_per_block))
            off += 2 * n * lay.bytes_per_block
        else:
            specs.append(SaveSpec(lay, np.asarray(ids), pool_ptr + off, None))
            off += n * lay.block_size_bytes
        off = (off + 255) // 256 * 256
    return specs, off


def save_noalloc(native, specs, stream):
    from pegaflow_b200.transfer import _save_array

    arr, keep = _save_array(specs)
    rc = native.lib.pf_save_blocks_noalloc(0, arr, len(specs), ctypes.c_void_p(stream))
    del keep
    return rc


@pytest.mark.parametrize("call_order", ["small_then_large", "large_then_small"])
def test_noalloc_save_matches_executor_save_on_consecutive_calls(cuda, native, call_order):
    torch = cuda
    from pegaflow_b200 import Executor, PinnedBuffer

    rng = np.random.default_rng(21)
    # Call A: mixed layouts in one staging slot. Call B: 24 MiB of KV-first
    # blocks, so the 8 MiB staging slot is refilled several times.
    call_a = ([kv(torch, (2, 64, 16, 2, 128), torch.bfloat16, 1), kv(torch, (64, 16, 4, 64), torch.float16, 2),
               kv(torch, (64,), torch.float32, 3), kv(torch, (2, 64, 5, 9), torch.uint8, 4)],
              [rng.permutation(64)[:40] for _ in range(4)])
    call_b = ([kv(torch, (2, 512, 16, 8, 128), torch.bfloat16, 5 + i) for i in range(2)],
              [rng.permutation(512)[:192] for _ in range(2)])
    calls = [call_a, call_b] if call_order == "small_then_large" else [call_b, call_a]

    ex = Executor(0)
    stream = torch.cuda.Stream()
    for tensors, ids_list in calls:
        probe, size = specs_for(tensors, ids_list, 0)
        ref_pool, pool = PinnedBuffer(size), PinnedBuffer(size)
        ref_pool.numpy()[:] = 0
        pool.numpy()[:] = 0xAB
        ref_specs, _ = specs_for(tensors, ids_list, ref_pool.ptr)
        ex.save(ref_specs)  # the existing entry point (pf_save_blocks)
        specs, _ = specs_for(tensors, ids_list, pool.ptr)
        native.check(save_noalloc(native, specs, stream.cuda_stream))
        stream.synchronize()
        # Compare only the bytes the saves own (regions between layers are padding).
        for r, s in zip(ref_specs, specs):
            lay = r.layout
            n = len(r.block_idx)
            unit = lay.bytes_per_block if lay.split else lay.block_size_bytes
            spans = [(r.k_dst - ref_pool.ptr, n * unit)]
            if lay.split:
                spans.append((r.v_dst - ref_pool.ptr, n * unit))
            for off, length in spans:
                np.testing.assert_array_equal(pool.numpy()[off:off + length], ref_pool.numpy()[off:off + length])


def test_noalloc_refuses_a_plan_beyond_its_scratch(cuda, native):
    torch = cuda
    from pegaflow_b200 import Layout, PinnedBuffer, SaveSpec

    nb = 300_000  # 300k block ids = 1.2 MB of plan > 1 MiB
    t = torch.zeros((nb, 16), dtype=torch.uint8, device="cuda")
    pool = PinnedBuffer(nb * 16)
    spec = SaveSpec(Layout.from_tensor(t), np.arange(nb), pool.ptr, None)
    rc = save_noalloc(native, [spec], 0)
    assert rc == native.PF_ERR_INVALID_ARGUMENT
    assert "exceeds the no-allocation limit" in native.lib.pf_last_error().decode()


def test_noalloc_save_of_unaligned_units_across_chunks(cuda, native, oracle):
    """45-byte units (a [2, nb, 5, 9] uint8 layer) over three 8 MiB staging
    chunks: chunk boundaries fall off the 256-byte slot alignment. Each chunk
    copies out only its own bytes, so every boundary matches the oracle (the
    copies once started at the aligned slot base and overwrote the previous
    chunk's last bytes with stale slot bytes)."""
    torch = cuda
    from pegaflow_b200 import Layout, PinnedBuffer, SaveSpec

    nb, n = 250_000, 200_000  # 2 x 200k x 45 B = 18 MB: three chunks
    t = kv(torch, (2, nb, 5, 9), torch.uint8, 31)
    lay = Layout.from_tensor(t)
    assert lay.split and lay.bytes_per_block == 45
    ids = np.random.default_rng(32).permutation(nb)[:n]
    pool = PinnedBuffer(2 * n * 45)
    pool.numpy()[:] = 0xAB
    stream = torch.cuda.Stream()
    native.check(save_noalloc(native, [SaveSpec(lay, ids, pool.ptr, pool.ptr + n * 45)], stream.cuda_stream))
    stream.synchronize()
    host = t.cpu().contiguous().view(-1).numpy()
    ol = oracle.Layout(lay.size_bytes, lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, lay.segments)
    k_ref, v_ref = oracle.np_save_layer(ol, host, ids)
    np.testing.assert_array_equal(pool.numpy()[: n * 45], k_ref)
    np.testing.assert_array_equal(pool.numpy()[n * 45:], v_ref)


def test_noalloc_takes_no_device_memory_after_warm_up(cuda, native):
    """The point of the entry point: after the warm-up call (no layers), which
    loads the library's device code and so reserves the fixed arrays, a
    multi-chunk save leaves the device's free memory exactly as it was. The
    callers it serves have already handed all free HBM to their own
    allocator, so a save that took any would fail there."""
    torch = cuda
    from pegaflow_b200 import PinnedBuffer

    stream = torch.cuda.Stream()
    native.check(native.lib.pf_save_blocks_noalloc(0, None, 0, ctypes.c_void_p(stream.cuda_stream)))
    rng = np.random.default_rng(41)
    tensors = [kv(torch, (2, 512, 16, 8, 128), torch.bfloat16, 50 + i) for i in range(2)]
    ids_list = [rng.permutation(512)[:192] for _ in range(2)]  # 24 MiB: three 8 MiB chunks
    _, size = specs_for(tensors, ids_list, 0)
    pool = PinnedBuffer(size)
    specs, _ = specs_for(tensors, ids_list, pool.ptr)
    torch.cuda.synchronize()
    for _ in range(2):
        free_before = torch.cuda.mem_get_info(0)[0]
        native.check(save_noalloc(native, specs, stream.cuda_stream))
        stream.synchronize()
        assert torch.cuda.mem_get_info(0)[0] == free_before
    k = specs[0]
    got = pool.numpy()[k.k_dst - pool.ptr:k.k_dst - pool.ptr + 192 * 32768]
    want = tensors[0][0, torch.as_tensor(ids_list[0], device="cuda")].contiguous().view(torch.uint8).cpu().numpy()
    np.testing.assert_array_equal(got, want.reshape(-1))
