"""The bulk kernel's bounded waits, run out on purpose.

The bulk (TMA) pack/unpack kernel waits on an mbarrier for each tile's bulk
load. Every such wait is bounded (1 s): if it runs out, the warp stops,
waits (bounded) for its other loads, and the kernel returns with a status
word set, which the executor turns into an error. The test hook
pf_executor_debug_stall_tile arms one tile's barrier without issuing its copy
(a barrier nothing completes: no fault, no hang), so the wait runs out. The
call must fail with the bounded-wait error within a few seconds, and the GPU
and the executor must stay usable: the next save moves the right bytes.
"""

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def kv(torch, shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("direction", ["save", "load"])
def test_bulk_wait_that_runs_out_fails_the_call_and_the_gpu_stays_usable(cuda, native, direction):
    torch = cuda
    from pegaflow_b200 import Executor, Layout, LoadSpec, PinnedBuffer, SaveSpec

    t = kv(torch, (2, 256, 16, 8, 128), 61)
    lay = Layout.from_tensor(t)
    n, seg = 64, lay.bytes_per_block
    perm = np.random.default_rng(62).permutation(256)
    src, dst = perm[:n], perm[n:2 * n]  # disjoint: a restore never overwrites a source
    pool = PinnedBuffer(2 * n * seg)
    save = SaveSpec(lay, src, pool.ptr, pool.ptr + n * seg)
    ks = np.arange(n, dtype=np.uint64) * seg + pool.ptr
    load = LoadSpec(lay, dst, ks, ks + n * seg)
    ex = Executor(0, copy_kernel="bulk")
    ex.save([save])  # the pool holds the source blocks
    torch.cuda.synchronize()

    native.check(native.lib.pf_executor_debug_stall_tile(ex._h, 37))
    t0 = time.perf_counter()
    with pytest.raises(native.PegaError) as err:
        ex.save([save]) if direction == "save" else ex.load([load])
    elapsed = time.perf_counter() - t0
    assert err.value.code == native.PF_ERR_STORAGE
    assert "gave up waiting" in str(err.value)
    assert 0.9 < elapsed < 30.0

    # Still usable: a normal round trip restores every block bit for bit.
    pool.numpy()[:] = 0
    ex.save([save])
    ex.load([load])
    torch.cuda.synchronize()
    si, di = torch.as_tensor(src, device="cuda"), torch.as_tensor(dst, device="cuda")
    assert torch.equal(t.index_select(1, di), t.index_select(1, si))
    want = t[0].index_select(0, si).contiguous().view(-1).view(torch.uint8).cpu().numpy()
    np.testing.assert_array_equal(pool.numpy()[: n * seg], want)
