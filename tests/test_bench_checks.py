"""bench.py's byte checks on the CPU: the helpers that decide `verified` in the
benchmark line must accept exactly a correct restore and a correct pool.

- scribble zeroes the destination blocks, so an untouched destination fails
  the restore check;
- restored accepts destination blocks equal to their sources and refuses a
  single flipped byte;
- pool_matches accepts the pool layout of lib.rs:639-679 (per layer, the K
  region then the V region, in block-list order) and refuses a pool with one
  wrong byte or with K and V swapped.
"""

import types

import numpy as np
import torch

import bench
from pegaflow_b200.ranks import block_lists


def kv_tensors(layers=3, nb=64, heads=2):
    g = torch.Generator().manual_seed(5)
    return [torch.randn((2, nb, 16, heads, 128), generator=g).to(torch.bfloat16) for _ in range(layers)]


def fake_pool(nbytes):
    arr = np.zeros(nbytes, np.uint8)
    return types.SimpleNamespace(ptr=arr.ctypes.data, numpy=lambda: arr, arr=arr)


def fill_pool(pool, tensors, saves, src):
    """Write the pool the way a correct save does."""
    si = torch.as_tensor(src)
    for t, sp in zip(tensors, saves):
        for kv, base in ((t[0], sp.k_dst), (t[1], sp.v_dst)):
            b = kv.index_select(0, si).contiguous().view(-1).view(torch.uint8).numpy()
            off = base - pool.ptr
            pool.arr[off:off + b.size] = b


def test_restore_check_needs_every_destination_byte():
    tensors = kv_tensors()
    src, dst = block_lists(64, 20, 0, "shuffled")
    assert not set(src) & set(dst)
    bench.scribble(torch, tensors, dst)
    assert not bench.restored(torch, tensors, src, dst)
    for t in tensors:
        t[:, torch.as_tensor(dst)] = t[:, torch.as_tensor(src)]
    assert bench.restored(torch, tensors, src, dst)
    tensors[1].view(torch.uint8).view(-1)[tensors[1][0, 0].numel() * 2 * int(dst[7]) + 3] ^= 1
    assert not bench.restored(torch, tensors, src, dst)


def test_pool_check_follows_the_reference_pool_layout():
    tensors = kv_tensors()
    src, dst = block_lists(64, 20, 0, "sorted")
    _, _, size = bench.executor_specs(tensors, src, dst, 0)
    pool = fake_pool(size)
    saves, _, _ = bench.executor_specs(tensors, src, dst, pool.ptr)
    fill_pool(pool, tensors, saves, src)
    assert bench.pool_matches(torch, tensors, saves, pool, src)
    # One wrong byte in the last layer's V region.
    last = saves[-1]
    pool.arr[last.v_dst - pool.ptr + 100] ^= 0xFF
    assert not bench.pool_matches(torch, tensors, saves, pool, src)
    pool.arr[last.v_dst - pool.ptr + 100] ^= 0xFF
    # K and V regions swapped in the first layer.
    first = saves[0]
    n = len(src) * first.layout.bytes_per_block
    k0, v0 = first.k_dst - pool.ptr, first.v_dst - pool.ptr
    k_bytes = pool.arr[k0:k0 + n].copy()
    pool.arr[k0:k0 + n] = pool.arr[v0:v0 + n]
    pool.arr[v0:v0 + n] = k_bytes
    assert not bench.pool_matches(torch, tensors, saves, pool, src)
