"""Connector host logic on CPU: scheduler metadata across chunked prefill,
save-segment identities, asynchronous lookups, the Sparse-Q span extension,
the in-process tensor-parallel lookup protocol, and the Store pipeline's
wait / publication / abort rules.  Mirrors the reference's
tests/test_connector_scheduler.py and tests/test_connector_writeback.py with
fakes for vLLM objects, streams and events (no GPU)."""

from __future__ import annotations

import threading
import time
from concurrent.futures import ThreadPoolExecutor
from types import SimpleNamespace

import pytest
import torch

connector_module = pytest.importorskip("cacheblend_b200.connector")
from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole  # noqa: E402

from cacheblend_b200 import registry  # noqa: E402
from cacheblend_b200.config import CacheBlendConfig  # noqa: E402
from cacheblend_b200.matcher import content_hash  # noqa: E402
from cacheblend_b200.storage import LocalPinnedCPUStore  # noqa: E402
from cacheblend_b200.store_path import StorePipeline  # noqa: E402
from cacheblend_b200.trace import PipelineTracer  # noqa: E402
from cacheblend_b200.types import BlendPlan, BlendSegment, SegmentId  # noqa: E402

CacheBlendConnectorV1 = connector_module.CacheBlendConnectorV1
RequestMetadata = connector_module.RequestMetadata
LocalStoreLookup = connector_module.LocalStoreLookup


def make_connector(**extra):
    connector = object.__new__(CacheBlendConnectorV1)
    connector.config = CacheBlendConfig.from_extra_config(
        {"chunk_size": 4, "strict_version_check": False, **extra}
    )
    connector.block_size = 2
    connector.engine_id = "test-engine"
    connector.model_scope = "model"
    connector.tp_size = 1
    connector._role = KVConnectorRole.SCHEDULER
    connector._init_state(KVConnectorRole.SCHEDULER)
    return connector


def output(new=(), cached=None, scheduled=None, preempted=None, finished=()):
    if cached is None:
        cached = SimpleNamespace(req_ids=[], resumed_req_ids=set(), new_block_ids=[],
                                 num_computed_tokens=[])
    return SimpleNamespace(scheduled_new_reqs=list(new), scheduled_cached_reqs=cached,
                           num_scheduled_tokens=scheduled or {}, finished_req_ids=set(finished),
                           preempted_req_ids=preempted)


def request(request_id, tokens, mm=()):
    return SimpleNamespace(request_id=request_id, prompt_token_ids=list(tokens),
                           _all_token_ids=list(tokens), lora_request=None, mm_features=list(mm),
                           prompt_embeds=None)


def test_slot_mapping_and_layer_order():
    assert connector_module._slot_mapping([3, 5], 4, 6).tolist() == [12, 13, 14, 15, 20, 21]
    names = ["model.layers.10.attn", "model.layers.2.attn", "model.layers.0.attn"]
    assert sorted(names, key=connector_module._layer_sort_key) == [
        "model.layers.0.attn", "model.layers.2.attn", "model.layers.10.attn"]


def test_metadata_tracks_full_blocks_across_chunked_prefill():
    connector = make_connector()
    req = request("r", range(10))
    connector._request_objects["r"] = req
    connector._plans["r"] = BlendPlan(0, 0, 0, ())
    first = SimpleNamespace(req_id="r", prompt_token_ids=req.prompt_token_ids,
                            block_ids=([3, 5, 7],), num_computed_tokens=4)
    metadata = connector.build_connector_meta(output([first], scheduled={"r": 2}))
    assert metadata.requests[0].save_end == 6
    assert metadata.requests[0].slot_mapping.tolist() == [6, 7, 10, 11, 14, 15]

    cached = SimpleNamespace(req_ids=["r"], resumed_req_ids=set(), new_block_ids=[([9],)],
                             num_computed_tokens=[6])
    metadata = connector.build_connector_meta(output(cached=cached, scheduled={"r": 2}))
    assert metadata.requests[0].plan is None
    assert metadata.requests[0].save_end == 8
    assert metadata.requests[0].slot_mapping.tolist() == [6, 7, 10, 11, 14, 15, 18, 19]


def test_preempted_request_is_resumed_with_new_blocks():
    connector = make_connector()
    req = request("p", range(8))
    connector._request_objects["p"] = req
    new = SimpleNamespace(req_id="p", prompt_token_ids=req.prompt_token_ids,
                          block_ids=([1, 2],), num_computed_tokens=0)
    connector.build_connector_meta(output([new], scheduled={"p": 4}))
    metadata = connector.build_connector_meta(output(preempted={"p"}))
    assert metadata.requests == []
    cached = SimpleNamespace(req_ids=["p"], resumed_req_ids={"p"}, new_block_ids=[([6, 7],)],
                             num_computed_tokens=[0])
    metadata = connector.build_connector_meta(output(cached=cached, scheduled={"p": 4}))
    assert metadata.requests[0].slot_mapping.tolist() == [12, 13, 14, 15]


def test_planned_load_is_emitted_once():
    connector = make_connector()
    req = request("l", range(12))
    plan = BlendPlan.from_segments(0, (BlendSegment(SegmentId("model", 1, 0, 4), 4),))
    connector._request_objects["l"] = req
    connector._plans["l"] = plan
    connector.update_state_after_alloc(req, None, plan.allocation_end)
    new = SimpleNamespace(req_id="l", prompt_token_ids=req.prompt_token_ids,
                          block_ids=([0, 1, 2, 3, 4, 5],), num_computed_tokens=0)
    metadata = connector.build_connector_meta(output([new], scheduled={"l": 11}))
    assert metadata.requests[0].plan == plan
    assert "l" not in connector._load_requests
    with pytest.raises(RuntimeError, match="missing CacheBlend plan"):
        connector.update_state_after_alloc(request("x", range(4)), None, 4)


def test_non_token_identified_request_is_not_saved():
    connector = make_connector()
    req = request("mm", [1, 2, 3], mm=[object()])
    connector._request_objects["mm"] = req
    new = SimpleNamespace(req_id="mm", prompt_token_ids=req.prompt_token_ids,
                          block_ids=([1, 2],), num_computed_tokens=0)
    metadata = connector.build_connector_meta(output([new], scheduled={"mm": 3}))
    assert not metadata.requests[0].save
    assert metadata.requests[0].save_end == 3
    assert connector.get_num_new_matched_tokens(req, 0) == (0, False)


def test_save_end_includes_decode_only_when_configured():
    connector = make_connector()
    req = request("d", range(6))
    req._all_token_ids = list(range(9))
    assert connector._save_end(req, 9, 9) == 6
    connector.config = CacheBlendConfig.from_extra_config(
        {"chunk_size": 4, "strict_version_check": False, "save_decode_cache": True})
    assert connector._save_end(req, 9, 9) == 9
    assert CacheBlendConnectorV1.requires_piecewise_for_cudagraph({"save_decode_cache": True})
    assert not CacheBlendConnectorV1.requires_piecewise_for_cudagraph({})


class CountingStore:
    def __init__(self):
        self.calls = []

    def begin_put(self, model_scope, source_start, tokens, num_layers):
        token_tuple = tuple(tokens)
        self.calls.append((model_scope, source_start, token_tuple, num_layers))
        return SegmentId(model_scope, content_hash(token_tuple), source_start, len(token_tuple))

    def begin_put_chunks(self, model_scope, first_start, tokens, count, num_layers):
        return [self.begin_put(model_scope, first_start + i * 4, tokens[first_start + i * 4 : first_start + (i + 1) * 4],
                               num_layers) for i in range(count)]


def test_save_segment_hashes_are_built_once_per_request():
    connector = make_connector()
    connector._store = CountingStore()
    connector._kv_caches = [object(), object()]
    meta = RequestMetadata("r", list(range(12)), torch.arange(12), None, True, 12)
    first = connector._request_save_segments(meta, 8)
    assert [start for start, _ in first] == [0, 4]
    assert len(connector._store.calls) == 2
    grown = connector._request_save_segments(meta, 12)
    assert [start for start, _ in grown] == [0, 4, 8]
    assert len(connector._store.calls) == 3
    assert connector._request_save_segments(meta, 12) == grown
    assert len(connector._store.calls) == 3
    assert connector._store.calls[1] == ("model", 4, (4, 5, 6, 7), 2)


def test_scheduler_lookup_is_submitted_and_polled_without_blocking(monkeypatch):
    connector = make_connector()
    connector._lookup_pool = ThreadPoolExecutor(max_workers=1)
    entered, release = threading.Event(), threading.Event()

    def lookup_plan(_request_id, _tokens, apc_prefix_tokens):
        entered.set()
        assert release.wait(timeout=5)
        return BlendPlan(apc_prefix_tokens, apc_prefix_tokens, 0, ())

    monkeypatch.setattr(connector, "_lookup_plan", lookup_plan)
    req = request("async", range(12))
    assert connector.get_num_new_matched_tokens(req, 0) == (None, True)
    assert entered.wait(timeout=2)
    assert connector.get_num_new_matched_tokens(req, 0) == (None, True)
    release.set()
    deadline = time.monotonic() + 2
    result = (None, True)
    while result[1] and time.monotonic() < deadline:
        result = connector.get_num_new_matched_tokens(req, 0)
        time.sleep(0.001)
    assert result == (0, False)
    connector._lookup_pool.shutdown(wait=True)


def test_short_prompt_skips_lookup_and_failed_lookup_recomputes(monkeypatch):
    connector = make_connector()
    connector._lookup_pool = ThreadPoolExecutor(max_workers=1)
    assert connector.get_num_new_matched_tokens(request("s", range(4)), 0) == (0, False)
    assert connector._plans["s"].allocation_end == 0

    def broken(*_args):
        raise ConnectionError("lookup down")

    monkeypatch.setattr(connector, "_lookup_plan", broken)
    req = request("f", range(12))
    assert connector.get_num_new_matched_tokens(req, 2) == (None, True)
    deadline = time.monotonic() + 2
    result = (None, True)
    while result[1] and time.monotonic() < deadline:
        result = connector.get_num_new_matched_tokens(req, 2)
    assert result == (0, False)
    assert connector._plans["f"] == BlendPlan(2, 2, 0, ())
    connector._lookup_pool.shutdown(wait=True)


class StaticLookup:
    def __init__(self, segments):
        self.segments = segments
        self.cancelled = []

    def lookup_and_prefetch(self, *_args):
        return list(self.segments)

    def cancel(self, request_id):
        self.cancelled.append(request_id)


def test_sparse_q_lookup_includes_trailing_query_tokens():
    connector = make_connector(selection_strategy="sparse_q", check_layers=[1], min_retrieve_tokens=0)
    segment = BlendSegment(SegmentId("model", content_hash((0, 1, 2, 3)), 0, 4), target_start=0)
    connector._lookup = StaticLookup([segment])
    plan = connector._lookup_plan("sparse", list(range(12)), 0)
    assert (plan.allocation_end, plan.hit_tokens, plan.gap_tokens) == (11, 4, 7)
    assert connector._lookup.cancelled == []


def test_gated_plan_is_cancelled():
    connector = make_connector(min_retrieve_tokens=64)
    segment = BlendSegment(SegmentId("model", 7, 0, 4), target_start=0)
    connector._lookup = StaticLookup([segment])
    assert connector._lookup_plan("g", list(range(12)), 0) == BlendPlan(0, 0, 0, ())
    assert connector._lookup.cancelled == ["g"]


def test_cancelled_lookup_returns_empty_plan():
    connector = make_connector(min_retrieve_tokens=0)
    connector._lookup = StaticLookup([BlendSegment(SegmentId("model", 7, 0, 4), 0)])
    connector._cancelled_lookup_ids.add("c")
    assert connector._lookup_plan("c", list(range(12)), 0) == BlendPlan(0, 0, 0, ())


def _committed_store(chunk, tokens, layers=2):
    store = LocalPinnedCPUStore(chunk, 1 << 20, pin_memory=False)
    sid = store.begin_put("model", 0, tokens, layers)
    for layer in range(layers):
        store.put_layer_host(sid, layer, torch.zeros(2, chunk, 1, 2))
    return store, sid


def test_local_lookup_intersects_ranks_and_pins():
    registry.clear_for_test()
    try:
        tokens = [5, 6, 7, 8]
        rank0, sid = _committed_store(4, tokens)
        rank1, _ = _committed_store(4, tokens)
        registry.register_store("e", 0, rank0)
        registry.register_store("e", 1, rank1)
        lookup = LocalStoreLookup("e")
        prompt = [1, 2] + tokens + [9]
        found = lookup.lookup_and_prefetch("req", "model", prompt, 2)
        assert found == (BlendSegment(sid, 2),)
        assert rank0.get_layer("req", found[0], 1).shape == (2, 4, 1, 2)
        assert rank1.get_layer("req", found[0], 0).shape == (2, 4, 1, 2)
        lookup.cancel("req")
        with pytest.raises(RuntimeError):
            rank1.get_layer("req", found[0], 0)
        # a rank without the chunk empties the intersection
        registry.register_store("e", 1, LocalPinnedCPUStore(4, 1 << 20, pin_memory=False))
        assert lookup.lookup_and_prefetch("req2", "model", prompt, 2) == ()
        with pytest.raises(RuntimeError):
            rank0.get_layer("req2", found[0], 0)
    finally:
        registry.clear_for_test()


def test_cleanup_releases_scheduler_state():
    connector = make_connector()
    connector._lookup = StaticLookup(())
    connector._lookup_pool = ThreadPoolExecutor(max_workers=1)
    req = request("z", range(12))
    connector._plans["z"] = BlendPlan(0, 0, 0, ())
    connector._request_objects["z"] = req
    assert connector.request_finished(req, []) == (False, None)
    connector._lookup_pool.shutdown(wait=True)
    assert "z" not in connector._plans and "z" not in connector._request_objects
    assert connector._lookup.cancelled == ["z"]


# ------------------------------------------------------------ store pipeline host logic
class RecordingStream:
    def __init__(self):
        self.synchronize_calls = 0

    def synchronize(self):
        self.synchronize_calls += 1


class RecordingEvent:
    def __init__(self):
        self.synchronize_calls = 0

    def synchronize(self):
        self.synchronize_calls += 1


class RecordingStore:
    def __init__(self, fail_at=None):
        self.layers, self.aborted, self.fail_at = [], [], fail_at

    def put_layer_host(self, segment_id, layer_id, tensor):
        if segment_id == self.fail_at:
            raise RuntimeError("publication failed")
        self.layers.append((segment_id, layer_id, tensor))
        return True

    def put_layers_host(self, segment_ids, layer_id, tensors):
        return [self.put_layer_host(sid, layer_id, t) for sid, t in zip(segment_ids, tensors)]

    def abort_put(self, segment_id):
        self.aborted.append(segment_id)


def bare_pipeline(store):
    pipeline = object.__new__(StorePipeline)
    pipeline.store = store
    pipeline.tracer = PipelineTracer("test")
    pipeline._lock = threading.Lock()
    pipeline._futures = set()
    pipeline._pending_counts = {}
    pipeline._staging = {"r": torch.empty(1)}
    pipeline._retired = [torch.empty(1)]
    pipeline._slot_cache = {"r": ((0, 0, 0, 0), torch.empty(1), torch.empty(1))}
    pipeline._layouts = {}
    pipeline._slots = threading.Semaphore(2)
    pipeline._pool = ThreadPoolExecutor(max_workers=1)
    pipeline.stream = RecordingStream()
    return pipeline


def test_wait_for_save_synchronizes_store_stream_and_drops_staging():
    pipeline = bare_pipeline(RecordingStore())
    assert pipeline.wait_for_save() == {}
    assert pipeline.stream.synchronize_calls == 1
    assert pipeline._staging == {} and pipeline._retired == [] and pipeline._slot_cache == {}
    pipeline._pool.shutdown()


def test_publication_views_chunks_and_counts_per_request():
    store = RecordingStore()
    pipeline = bare_pipeline(store)
    host = torch.arange(2 * 2 * 4 * 3).reshape(2, 2, 4, 3)  # [chunks, K/V, chunk, row]
    event = RecordingEvent()
    future = pipeline._pool.submit(pipeline._publish_after_event, event,
                                   [("a", 5, 4), ("b", 5, 4)], host, "r", None)
    with pipeline._lock:
        pipeline._futures.add(future)
        pipeline._pending_counts["r"] = 1
    assert pipeline.wait_for_save() == {"r": 1}
    assert event.synchronize_calls == 1
    assert [(sid, layer) for sid, layer, _ in store.layers] == [("a", 5), ("b", 5)]
    assert torch.equal(store.layers[1][2], host[1])
    assert store.layers[1][2].data_ptr() == host[1].data_ptr()  # a view, no host copy
    pipeline._pool.shutdown()


def test_async_publish_aborts_the_whole_batch_on_failure():
    store = RecordingStore(fail_at="segment-b")
    pipeline = bare_pipeline(store)
    host = torch.zeros(2, 2, 2, 4)
    assert not pipeline._publish_after_event(RecordingEvent(),
                                             [("segment-a", 3, 2), ("segment-b", 3, 2)], host)
    assert store.aborted == ["segment-a", "segment-b"]
    pipeline._pool.shutdown()
