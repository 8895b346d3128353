"""The vLLM connector end to end on a GPU: scheduler side and worker side
over the engine server (a separate process mapping this process's KV caches
by CUDA IPC). A request is prefilled and saved layer by layer; a second
request with the same prefix is matched by the scheduler and restored into
other blocks, either inside the forward (layer-wise: wait_for_layer_load)
or asynchronously (get_finished), and the restored bytes equal the saved."""

import time
import types

import pytest

pytestmark = pytest.mark.gpu


def gen(torch, shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(torch.bfloat16).cuda()


def scheduled(req_id, tokens):
    return types.SimpleNamespace(scheduled_new_reqs=[types.SimpleNamespace(req_id=req_id)],
                                 num_scheduled_tokens={req_id: tokens},
                                 scheduled_cached_reqs=types.SimpleNamespace(req_ids=[], new_block_ids=[]))


def wait_for(fn, what, timeout=60.0):
    t0 = time.time()
    while True:
        v = fn()
        if v:
            return v
        assert time.time() - t0 < timeout, what
        time.sleep(0.002)


@pytest.mark.parametrize("layerwise", [True, False])
def test_prefill_save_then_restore_through_connector(cuda, engine_server, layerwise):
    torch = cuda
    from pegaflow_b200.connector import ConnectorContext, SchedulerSide, WorkerSide

    client, _ = engine_server()
    names = [f"model.layers.{i}.self_attn" for i in range(4)]
    caches = {n: gen(torch, (2, 64, 16, 8, 128), 10 + i) for i, n in enumerate(names)}
    ctx = ConnectorContext("inst", "ns", 16, len(names), 1, 0, 0, client, layerwise)
    sched, worker = SchedulerSide(ctx), WorkerSide(ctx)
    try:
        worker.register_kv_caches(caches)
        fwd = types.SimpleNamespace(no_compile_layers={n: types.SimpleNamespace(kv_cache=[caches[n]])
                                                       for n in names})
        attn = types.SimpleNamespace(block_table=object())
        hashes = [f"prefix-{i}".encode() for i in range(10)]

        # Request A: nothing cached; prefill 10 blocks and save them.
        req_a = types.SimpleNamespace(request_id="A", block_hashes=hashes, num_tokens=160)
        assert sched.get_num_new_matched_tokens(req_a, 0) == (0, False)
        src = [3, 7, 1, 9, 20, 33, 40, 41, 42, 63]
        sched.update_state_after_alloc(req_a, types.SimpleNamespace(get_block_ids=lambda: (src,)), 0)
        meta = sched.build_connector_meta(scheduled("A", 160))
        assert meta.save_intents["A"].block_ids == tuple(src)
        worker.start_load_kv(meta, fwd)
        for n in names:
            worker.save_kv_layer(meta, n, caches[n], attn)
        worker.wait_for_save()
        sending = wait_for(lambda: worker.get_finished({"A"})[0], "save of A did not complete")
        assert sending == {"A"}

        # Request B: the same 10 blocks plus one new block.
        req_b = types.SimpleNamespace(request_id="B", block_hashes=hashes + [b"suffix"], num_tokens=176)
        tokens, is_async = sched.get_num_new_matched_tokens(req_b, 0)
        assert (tokens, is_async) == (160, not layerwise)
        dst = [50, 51, 52, 53, 54, 55, 56, 57, 58, 59, 60]
        sched.update_state_after_alloc(req_b, types.SimpleNamespace(get_block_ids=lambda: (dst,)), 160)
        meta = sched.build_connector_meta(scheduled("B", 16))
        assert meta.load_intents["B"].block_ids == tuple(dst[:10])
        before = {n: t.clone() for n, t in caches.items()}
        src_t, dst_t = torch.tensor(src, device="cuda"), torch.tensor(dst[:10], device="cuda")
        worker.start_load_kv(meta, fwd)
        if layerwise:
            # Each layer's bytes are in place once its wait returns.
            for n in names:
                worker.wait_for_layer_load(n)
                assert torch.equal(caches[n].index_select(1, dst_t), before[n].index_select(1, src_t)), n
            # Layer-wise loads are not reported to vLLM; get_finished still
            # retires them once the whole task is done.
            def retired():
                assert worker.get_finished(set()) == (None, None)
                return not worker._loads

            wait_for(retired, "load bookkeeping did not settle")
        else:
            recving = wait_for(lambda: worker.get_finished(set())[1], "async load of B did not complete")
            assert recving == {"B"}
            torch.cuda.synchronize()
            for n in names:
                assert torch.equal(caches[n].index_select(1, dst_t), before[n].index_select(1, src_t)), n
    finally:
        worker.shutdown()
