"""Paged-to-paged block handoff between GPUs (prefill -> decode) over NVLink,
pull and push, checked byte for byte: destination block dst[i] of every layer
equals source block src[i]; everything else is untouched. The same-device
case (peer == this GPU) runs on one GPU; the cross-GPU case needs two."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def kv(torch, shape, seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(torch.bfloat16).to(device)


def run_handoff(torch, src_dev, dst_dev, push, nb_src=96, nb_dst=128, layers=3, n=40, dup=False):
    from pegaflow_b200 import Executor, Layout, P2PSpec

    srcs = [kv(torch, (2, nb_src, 16, 8, 128), 10 + i, f"cuda:{src_dev}") for i in range(layers)]
    srcs.append(kv(torch, (nb_src, 16, 4, 64), 99, f"cuda:{src_dev}"))  # a blocks-first layer
    dsts = [kv(torch, (2, nb_dst, 16, 8, 128), 50 + i, f"cuda:{dst_dev}") for i in range(layers)]
    dsts.append(kv(torch, (nb_dst, 16, 4, 64), 98, f"cuda:{dst_dev}"))
    rng = np.random.default_rng(3)
    src_ids = rng.permutation(nb_src)[:n]
    dst_ids = rng.permutation(nb_dst)[:n]
    if dup:
        dst_ids[5] = dst_ids[2]  # block dst_ids[2] receives src_ids[5] (the later one)
    before = [d.clone() for d in dsts]
    specs = [P2PSpec(Layout.from_tensor(s), Layout.from_tensor(d), src_ids, dst_ids) for s, d in zip(srcs, dsts)]
    ex = Executor(src_dev if push else dst_dev)
    torch.cuda.synchronize(src_dev)
    torch.cuda.synchronize(dst_dev)
    ex.p2p(specs, dst_dev if push else src_dev, push=push)
    torch.cuda.synchronize(src_dev)
    torch.cuda.synchronize(dst_dev)
    last = {}
    for i, d in enumerate(dst_ids):
        last[int(d)] = int(src_ids[i])
    for s, d, b in zip(srcs, dsts, before):
        expect = b.clone()
        sc = s.to(f"cuda:{dst_dev}")
        for dd, ss in last.items():
            if expect.dim() == 5:
                expect[:, dd] = sc[:, ss]
            else:
                expect[dd] = sc[ss]
        assert torch.equal(d, expect)
    assert ex.stats()["bytes_p2p"] > 0


@pytest.mark.parametrize("push", [False, True])
def test_same_device_cache_to_cache(cuda, push):
    run_handoff(cuda, 0, 0, push, dup=True)


@pytest.mark.parametrize("push", [False, True])
def test_two_gpu_handoff(cuda, push):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    run_handoff(cuda, 0, 1, push)
    run_handoff(cuda, 1, 0, push, dup=True)


def test_copies_inside_one_tensor_need_disjoint_blocks(cuda):
    """Source and destination in the same tensor: a block that one pair reads
    and another writes would race between warps, so it is refused before any
    launch; disjoint blocks copy normally."""
    torch = cuda
    from pegaflow_b200 import Executor, Layout, P2PSpec

    a = kv(torch, (2, 32, 16, 8, 128), 3, "cuda:0")
    lay = Layout.from_tensor(a)
    before = a.clone()
    with pytest.raises(RuntimeError, match="overlap"):
        Executor(0).p2p([P2PSpec(lay, lay, np.array([1, 2, 3]), np.array([3, 4, 5]))], 0)
    torch.cuda.synchronize()
    assert torch.equal(a, before)
    Executor(0).p2p([P2PSpec(lay, lay, np.array([1, 2, 3]), np.array([10, 11, 31]))], 0)
    torch.cuda.synchronize()
    expect = before.clone()
    expect[:, [10, 11, 31]] = before[:, [1, 2, 3]]
    assert torch.equal(a, expect)


def test_mismatched_layouts_are_refused(cuda):
    torch = cuda
    from pegaflow_b200 import Executor, Layout, P2PSpec

    a = kv(torch, (2, 16, 16, 8, 128), 1, "cuda:0")
    b = kv(torch, (2, 16, 16, 4, 128), 2, "cuda:0")
    with pytest.raises(RuntimeError, match="layouts differ"):
        Executor(0).p2p([P2PSpec(Layout.from_tensor(a), Layout.from_tensor(b), np.array([1]), np.array([2]))], 0)
    with pytest.raises(RuntimeError, match="out of range"):
        Executor(0).p2p([P2PSpec(Layout.from_tensor(a), Layout.from_tensor(a), np.array([16]), np.array([2]))], 0)
