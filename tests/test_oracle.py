"""Pins the oracle (CPU only): two independent restatements agree, the library's
host-side checks agree with the oracle, and layouts derived by the reference's
own connector code (tests/golden/registration.json) are reproduced."""

import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def random_layouts(rng, count):
    out = []
    for _ in range(count):
        kind = rng.integers(0, 5)
        nb = int(rng.integers(1, 40))
        bpb = int(rng.choice([4, 16, 48, 100, 512, 4096, 5000]))
        if kind == 0:  # blocks-first
            out.append(dict(num_blocks=nb, bytes_per_block=bpb, kv_stride_bytes=0, segments=1, size=nb * bpb))
        elif kind == 1:  # KV-first split
            stride = nb * bpb
            out.append(dict(num_blocks=nb, bytes_per_block=bpb, kv_stride_bytes=stride, segments=2, size=2 * stride))
        elif kind == 2:  # interleaved K/V: contiguous with 2 segments
            out.append(dict(num_blocks=nb, bytes_per_block=bpb, kv_stride_bytes=bpb, segments=2, size=(nb + 1) * bpb))
        elif kind == 3:  # 3 segments, strided
            stride = nb * bpb + 64
            out.append(dict(num_blocks=nb, bytes_per_block=bpb, kv_stride_bytes=stride, segments=3,
                            size=2 * stride + nb * bpb))
        else:  # 2 segments with stride < bpb (overlapping, accepted by the reference)
            stride = max(1, bpb // 2)
            out.append(dict(num_blocks=nb, bytes_per_block=bpb, kv_stride_bytes=stride, segments=2,
                            size=(nb - 1) * bpb + stride + bpb))
    return out


def test_oracle_save_matches_numpy_twin(oracle):
    rng = np.random.default_rng(0)
    for spec in random_layouts(rng, 60):
        L = oracle.Layout(spec["size"], spec["num_blocks"], spec["bytes_per_block"], spec["kv_stride_bytes"],
                          spec["segments"])
        oracle.validate_layout(L, "x")
        gpu = rng.integers(0, 256, L.size_bytes, dtype=np.uint8)
        n = int(rng.integers(0, L.num_blocks + 1))
        ids = rng.permutation(L.num_blocks)[:n]
        k_ref, v_ref = oracle.np_save_layer(L, gpu, ids)
        if L.split:
            k = np.zeros(n * L.bytes_per_block, np.uint8)
            v = np.zeros(n * L.bytes_per_block, np.uint8)
            copies = oracle.save_layer(L, gpu, ids, k, v)
            assert copies == 2 * n
            np.testing.assert_array_equal(k, k_ref)
            np.testing.assert_array_equal(v, v_ref)
        else:
            out = np.zeros(n * L.block_size_bytes, np.uint8)
            copies = oracle.save_layer(L, gpu, ids, out, None)
            assert copies == (n if L.contiguous else n * L.segments)
            np.testing.assert_array_equal(out, k_ref)


def test_oracle_load_matches_numpy_twin_and_merges_runs(oracle):
    rng = np.random.default_rng(1)
    for spec in random_layouts(rng, 60):
        L = oracle.Layout(spec["size"], spec["num_blocks"], spec["bytes_per_block"], spec["kv_stride_bytes"],
                          spec["segments"])
        n = int(rng.integers(0, L.num_blocks + 1))
        ids = rng.permutation(L.num_blocks)[:n]
        if not L.split and not L.contiguous:
            ids = ids[ids + L.segments <= L.num_blocks]  # the non-split load copies block_size at segment 0
            n = len(ids)
        unit = L.bytes_per_block if L.split else L.block_size_bytes
        pool = rng.integers(0, 256, max(1, 2 * n * unit), dtype=np.uint8)
        base = pool.ctypes.data
        k_src = [base + i * unit for i in range(n)]
        v_src = [base + n * unit + i * unit for i in range(n)] if L.split else None
        gpu_a = rng.integers(0, 256, L.size_bytes, dtype=np.uint8)
        gpu_b = gpu_a.copy()
        runs = oracle.load_layer(L, gpu_a, ids, k_src, v_src)
        kb = [pool[i * unit:(i + 1) * unit] for i in range(n)]
        vb = [pool[n * unit + i * unit:n * unit + (i + 1) * unit] for i in range(n)] if L.split else None
        oracle.np_load_layer(L, gpu_b, ids, kb, vb)
        np.testing.assert_array_equal(gpu_a, gpu_b)
        # transfer.rs:134-177: runs = maximal stretches where the GPU offset and
        # the host pointer both advance by one unit.
        def count_runs(goffs, hosts):
            return sum(1 for i in range(len(goffs))
                       if i == 0 or goffs[i] != goffs[i - 1] + unit or hosts[i] != hosts[i - 1] + unit)

        expect = count_runs([oracle.segment_offset(L, int(b), 0) for b in ids], k_src)
        if L.split:
            expect += count_runs([oracle.segment_offset(L, int(b), 1) for b in ids], v_src)
        assert runs == expect


def test_sorted_ids_from_one_batch_merge_into_one_run_per_segment(oracle):
    """cfg2's sorted-contiguous case: 640 ids 0..639 from one save batch -> 1 K
    run + 1 V run per layer (transfer.rs:116-198)."""
    nb, bpb = 1024, 32768 // 64
    L = oracle.Layout(2 * nb * bpb, nb, bpb, nb * bpb, 2)
    gpu = np.zeros(L.size_bytes, np.uint8)
    pool = np.arange(2 * 640 * bpb, dtype=np.uint64).astype(np.uint8)
    base = pool.ctypes.data
    runs = oracle.load_layer(L, gpu, list(range(640)), [base + i * bpb for i in range(640)],
                             [base + (640 + i) * bpb for i in range(640)])
    assert runs == 2
    rng = np.random.default_rng(3)
    shuffled = rng.permutation(nb)[:640]
    runs = oracle.load_layer(L, gpu, shuffled, [base + i * bpb for i in range(640)],
                             [base + (640 + i) * bpb for i in range(640)])
    assert runs > 2 * 600  # shuffled destinations break almost every run


def _layer_desc(native, spec):
    return native.LayerDesc(0x10000, spec["size"], spec["num_blocks"], spec["bytes_per_block"],
                            spec["kv_stride_bytes"], spec["segments"])


BAD_LAYOUTS = [
    dict(size=100, num_blocks=0, bytes_per_block=4, kv_stride_bytes=0, segments=1),
    dict(size=100, num_blocks=1, bytes_per_block=0, kv_stride_bytes=0, segments=1),
    dict(size=100, num_blocks=1, bytes_per_block=4, kv_stride_bytes=0, segments=0),
    dict(size=100, num_blocks=2, bytes_per_block=4, kv_stride_bytes=0, segments=2),
    dict(size=100, num_blocks=2, bytes_per_block=2**63, kv_stride_bytes=1, segments=2),
    dict(size=100, num_blocks=2**62, bytes_per_block=8, kv_stride_bytes=0, segments=1),
    dict(size=100, num_blocks=2, bytes_per_block=8, kv_stride_bytes=2**63, segments=3),
    dict(size=2**64 - 1, num_blocks=2**61, bytes_per_block=4, kv_stride_bytes=2**63, segments=2),
    dict(size=2**64 - 1, num_blocks=2, bytes_per_block=2**63, kv_stride_bytes=2**62, segments=2),
    dict(size=99, num_blocks=10, bytes_per_block=10, kv_stride_bytes=0, segments=1),
    dict(size=100, num_blocks=10, bytes_per_block=10, kv_stride_bytes=0, segments=1),
]


@pytest.mark.parametrize("spec", BAD_LAYOUTS)
def test_library_layout_checks_match_oracle(native, oracle, spec):
    from ctypes import byref

    L = oracle.Layout(spec["size"], spec["num_blocks"], spec["bytes_per_block"], spec["kv_stride_bytes"],
                      spec["segments"])
    try:
        oracle.validate_layout(L, "layer.x")
        expect = None
    except oracle.OracleError as e:
        expect = str(e)
    rc = native.lib.pf_layer_validate(byref(_layer_desc(native, spec)), b"layer.x")
    got = None if rc == 0 else native.lib.pf_last_error().decode()
    assert got == expect


def test_library_segment_offset_matches_oracle(native, oracle):
    from ctypes import byref, c_uint64

    rng = np.random.default_rng(4)
    specs = random_layouts(rng, 40) + [dict(size=2**64 - 1, num_blocks=2**40, bytes_per_block=2**30,
                                            kv_stride_bytes=2**62, segments=3)]
    for spec in specs:
        L = oracle.Layout(spec["size"], spec["num_blocks"], spec["bytes_per_block"], spec["kv_stride_bytes"],
                          spec["segments"])
        for b in [0, 1, spec["num_blocks"] - 1, spec["num_blocks"], spec["num_blocks"] + 7, 2**62]:
            for s in range(spec["segments"] + 1):
                try:
                    expect = oracle.segment_offset(L, b, s)
                except oracle.OracleError as e:
                    expect = "storage error: " + str(e)
                out = c_uint64()
                rc = native.lib.pf_segment_offset(byref(_layer_desc(native, spec)), b, s, byref(out))
                got = out.value if rc == 0 else native.lib.pf_last_error().decode()
                assert got == expect, (spec, b, s)


def test_registration_golden_layouts(native, oracle):
    """Layouts the reference's own worker connector derives (worker.py:100-115)
    for the benchmark shapes are reproduced by Layout.from_tensor."""
    import torch

    from pegaflow_b200 import Layout

    cases = json.loads((GOLDEN / "registration.json").read_text())
    assert len(cases) >= 8
    dtypes = {1: torch.uint8, 2: torch.bfloat16, 4: torch.float32}
    for c in cases:
        t = torch.empty(c["shape"], dtype=dtypes[c["element_size"]], device="meta")
        assert list(t.stride()) == c["stride"]
        lay = Layout.from_tensor(t)
        assert (lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, lay.segments) == (
            c["num_blocks"], c["bytes_per_block"], c["kv_stride_bytes"], c["segments"]), c["case"]
        # The layout is valid for a tensor of exactly that size, for both checkers.
        L = oracle.Layout(lay.size_bytes, lay.num_blocks, lay.bytes_per_block, lay.kv_stride_bytes, lay.segments)
        oracle.validate_layout(L, c["case"])
        from pegaflow_b200 import validate

        validate(lay, c["case"])


def test_save_batch_golden_is_self_consistent():
    """The reference connector groups per-layer tasks by layer, concatenating the
    save intents of every task of that layer, skipping tasks without a block
    table and intents without blocks (worker.py:372-402)."""
    g = json.loads((GOLDEN / "save_batches.json").read_text())
    (rpc,) = g["rpc"]
    layers = [s[0] for s in rpc["saves"]]
    assert layers == ["layer.0", "layer.1"]
    ids0 = rpc["saves"][0][1]
    assert ids0 == [5, 9, 2, 7, -1] * 2  # layer.0 appears in two tasks
    assert rpc["saves"][1][1] == [5, 9, 2, 7, -1]
