"""Engine host logic on a plain-memory pool (CPU only): the checks and errors
of PegaEngine (pegaflow-core/src/lib.rs) against the oracle's EngineModel."""

import numpy as np
import pytest

from pegaflow_b200 import PegaEngine, PyLoadState


@pytest.fixture
def engine(native):
    e = PegaEngine(1 << 20, pool_kind="host")
    yield e
    e.close()


def split_layout(nb=16, bpb=4096):
    return dict(size_bytes=2 * nb * bpb, num_blocks=nb, bytes_per_block=bpb, kv_stride_bytes=nb * bpb, segments=2)


def reg(e, inst="i", layer="L0", device=0, tp_rank=0, tp_size=1, num_layers=2, ns="ns", **lay):
    lay = lay or split_layout()
    e.register_context_layer(inst, ns, device, layer, 0x7000_0000, lay["size_bytes"], lay["num_blocks"],
                             lay["bytes_per_block"], lay["kv_stride_bytes"], lay["segments"], tp_rank, tp_size,
                             num_layers)


def model_reg(m, inst="i", layer="L0", device=0, tp_rank=0, tp_size=1, num_layers=2, ns="ns", **lay):
    from oracle.oracle import Layout

    lay = lay or split_layout()
    L = Layout(lay["size_bytes"], lay["num_blocks"], lay["bytes_per_block"], lay["kv_stride_bytes"], lay["segments"])
    m.register_context_layer(inst, ns, device, layer, np.zeros(L.size_bytes, np.uint8), L, tp_rank, tp_size,
                             num_layers)


def both_raise(fn_engine, fn_model, oracle):
    with pytest.raises(RuntimeError) as ei:
        fn_engine()
    with pytest.raises(oracle.OracleError) as em:
        fn_model()
    assert str(ei.value) == str(em.value)
    return str(ei.value)


def test_registration_errors_match_model(engine, oracle):
    m = oracle.EngineModel()
    bad = [
        dict(size_bytes=100, num_blocks=0, bytes_per_block=4, kv_stride_bytes=0, segments=1),
        dict(size_bytes=100, num_blocks=4, bytes_per_block=4, kv_stride_bytes=0, segments=2),
        dict(size_bytes=10, num_blocks=4, bytes_per_block=4, kv_stride_bytes=0, segments=1),
    ]
    for lay in bad:
        both_raise(lambda: reg(engine, **lay), lambda: model_reg(m, **lay), oracle)
    msg = both_raise(lambda: reg(engine, device=-1), lambda: model_reg(m, device=-1), oracle)
    assert msg == "invalid argument: device_id must be >= 0"


def test_topology_mismatch(engine, oracle):
    m = oracle.EngineModel()
    reg(engine)
    model_reg(m)
    msg = both_raise(lambda: reg(engine, layer="L1", tp_size=2), lambda: model_reg(m, layer="L1", tp_size=2), oracle)
    assert msg.startswith("topology mismatch: instance i exists with layers=2, tp=1")


def test_unregister_and_missing_instance(engine):
    reg(engine)
    engine.unregister_instance("i")
    with pytest.raises(RuntimeError, match="^instance i not found$"):
        engine.unregister_instance("i")
    with pytest.raises(RuntimeError, match="^instance nope not found$"):
        engine.count_prefix_hit_blocks("nope", [b"a"])


def test_prefix_count_on_empty_cache_counts_misses(engine):
    reg(engine)
    assert engine.count_prefix_hit_blocks("i", [b"a", b"b", b"c"]) == 0
    assert engine.metrics()["cache_block_misses"] == 3


def test_save_argument_errors_match_model(engine, oracle):
    m = oracle.EngineModel()
    reg(engine)
    model_reg(m)
    cases = [
        ("nope", 0, 0, [("L0", [1], [b"h"])]),            # InstanceMissing
        ("i", 0, 3, [("L0", [1], [b"h"])]),               # WorkerMissing
        ("i", 0, 0, [("Lx", [1], [b"h"])]),               # unknown layer
        ("i", 5, 0, [("L0", [1], [b"h"])]),               # tp_rank out of range
        ("i", 0, 0, [("L0", [99], [b"h"])]),              # block out of range
    ]
    for inst, rank, dev, saves in cases:
        both_raise(lambda: engine.batch_save_kv_blocks(inst, rank, dev, saves),
                   lambda: m.batch_save(inst, rank, dev, saves), oracle)
    with pytest.raises(RuntimeError, match="block_ids length 2 does not match block_hashes 1"):
        engine.batch_save_kv_blocks("i", 0, 0, [("L0", [1, 2], [b"h"])])


def test_save_of_only_negative_ids_is_a_no_op(engine):
    reg(engine)
    engine.batch_save_kv_blocks("i", 0, 0, [("L0", [-1, -5], [b"a", b"b"])])
    assert engine.metrics()["save_calls"] == 0


def test_save_needing_a_transfer_fails_loudly_without_gpu(engine):
    reg(engine)
    with pytest.raises(RuntimeError, match="failed to initialize CUDA"):
        engine.batch_save_kv_blocks("i", 0, 0, [("L0", [1], [b"a"])])


def test_load_errors_set_load_state_error(engine):
    reg(engine)
    s = PyLoadState()
    with pytest.raises(RuntimeError, match=r"missing KV block hash at index 0 \(namespace=ns, hash_len=1\)"):
        engine.batch_load_kv_blocks("i", 0, 0, s.shm_name(), ["L0"], [1], [b"a"])
    assert s.get_state() == -1 and s.is_ready()
    s2 = PyLoadState()
    with pytest.raises(RuntimeError, match="^instance x not found$"):
        engine.batch_load_kv_blocks("x", 0, 0, s2.shm_name(), ["L0"], [1], [b"a"])
    assert s2.get_state() == -1
    s3 = PyLoadState()
    with pytest.raises(RuntimeError, match="^device 4 not found in instance i$"):
        engine.batch_load_kv_blocks("i", 0, 4, s3.shm_name(), ["L0"], [1], [b"a"])
    assert s3.get_state() == -1


def test_load_with_bad_shm_name_is_a_storage_error(engine):
    reg(engine)
    with pytest.raises(RuntimeError, match="^storage error: LoadState: failed to open shared memory"):
        engine.batch_load_kv_blocks("i", 0, 0, "pega_load_does_not_exist", ["L0"], [1], [b"a"])


def test_load_with_no_blocks_completes_immediately(engine):
    reg(engine)
    s = PyLoadState()
    engine.batch_load_kv_blocks("i", 0, 0, s.shm_name(), ["L0"], [], [])
    assert s.get_state() == 1
    layered = PyLoadState(1)
    engine.batch_load_kv_blocks("i", 0, 0, layered.shm_name(), ["L0"], [-1], [])
    assert layered.get_state() == 1 and layered.layer_ready(0)
