"""Scheduler side of the vLLM connector: prefix lookups, load/save intents.

Same decisions as the reference scheduler (python/pegaflow/connector/
scheduler.py:35-268): the hit count is the engine's contiguous prefix of
sealed blocks; at least one token is always left for vLLM to compute; loads
are asynchronous (vLLM waits for get_finished) unless the connector runs in
layer-wise mode, where the load happens inside the forward.
"""

from __future__ import annotations

from typing import Optional

from .state import ConnectorContext, LoadIntent, PegaConnectorMetadata, RequestTracker, log


class SchedulerSide:
    def __init__(self, ctx: ConnectorContext):
        self._ctx = ctx
        self._trackers: dict[str, RequestTracker] = {}
        self._pending_loads: dict[str, LoadIntent] = {}
        self._held: set = set()

    def _tracker(self, request) -> RequestTracker:
        t = self._trackers.get(request.request_id)
        if t is None:
            t = RequestTracker(request.request_id, list(request.block_hashes), self._ctx.block_size,
                               self._ctx.num_layers)
            self._trackers[request.request_id] = t
        return t

    def _hit_blocks(self, hashes) -> Optional[int]:
        r = self._ctx.engine_client.query(self._ctx.instance_id, list(hashes))
        if not r.get("ok", False):
            raise RuntimeError(f"Query failed: {r.get('message', 'unknown error')}")
        if r.get("prefetch_state") == "loading":
            return None  # blocks on their way from a lower tier: ask again later
        return r.get("hit_blocks", 0)

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> tuple:
        tracker = self._tracker(request)
        hit = self._hit_blocks(request.block_hashes)
        if hit is None:
            return None, False
        tracker.on_lookup(hit, num_computed_tokens // self._ctx.block_size)
        tokens = hit * self._ctx.block_size - num_computed_tokens
        if tokens <= 0:
            return 0, False
        tokens = min(tokens, request.num_tokens - 1)  # vLLM must compute at least one token
        log.info("request %s: %d cached blocks, %d tokens to load", request.request_id, hit, tokens)
        return tokens, not self._ctx.layerwise

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        tracker = self._trackers.get(request.request_id)
        if tracker is None:
            return
        tracker.on_alloc(list(blocks.get_block_ids()[0]) if blocks else [], num_external_tokens)
        intent = tracker.consume_load_intent()  # always consumed: no stale window after preemption
        if intent is not None:
            self._pending_loads[request.request_id] = intent

    def build_connector_meta(self, scheduler_output) -> PegaConnectorMetadata:
        loads, self._pending_loads = self._pending_loads, {}
        saves = {}
        for req in scheduler_output.scheduled_new_reqs:
            tracker = self._trackers.get(req.req_id)
            if tracker is None:
                continue
            tracker.on_scheduled(scheduler_output.num_scheduled_tokens.get(req.req_id, 0))
            if req.req_id not in loads:
                intent = tracker.consume_load_intent()
                if intent is not None:
                    loads[req.req_id] = intent
            s = tracker.consume_save_intent()
            if s is not None:
                saves[req.req_id] = s
        cached = scheduler_output.scheduled_cached_reqs
        for i, req_id in enumerate(cached.req_ids):
            tracker = self._trackers.get(req_id)
            if tracker is None:
                continue
            tracker.on_scheduled(scheduler_output.num_scheduled_tokens.get(req_id, 0))
            new_ids = cached.new_block_ids[i]
            if new_ids:
                tracker.on_alloc(list(new_ids[0]), 0)
            s = tracker.consume_save_intent()
            if s is not None:
                saves[req_id] = s
        return PegaConnectorMetadata(load_intents=loads, save_intents=saves)

    def update_connector_output(self, connector_output) -> None:
        for req_id in connector_output.finished_sending or []:
            tracker = self._trackers.get(req_id)
            if tracker is None:
                continue
            tracker.saved_layers = tracker.total_layers
            self._held.discard(req_id)
            if tracker.is_done():
                del self._trackers[req_id]

    def request_finished(self, request, block_ids) -> tuple:
        tracker = self._trackers.get(request.request_id)
        if tracker is not None:
            tracker.on_finished()
            if tracker.should_hold_blocks():  # keep blocks until their save lands
                self._held.add(request.request_id)
                return True, None
        return False, None
