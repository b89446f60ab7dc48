"""Host-side logic of the product (no GPU): config schema, plan types, store
lifecycle (replayed against the reference's recorded op sequence), content
fingerprints, the recompute budget and the Sparse-Q masks."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.config import CacheBlendConfig
from cacheblend_b200.matcher import content_hash, window_hashes
from cacheblend_b200.selection import recompute_budget, sparse_q_masks
from cacheblend_b200.storage import LocalPinnedCPUStore
from cacheblend_b200.types import BlendPlan, BlendSegment, SegmentId


def test_config_matches_reference_contract():
    # reference tests/test_config_registry.py:13-56
    config = CacheBlendConfig.from_extra_config(
        {"check_layers": 2, "recompute_ratios": 0.25, "strict_version_check": False}
    )
    assert config.check_layers == (2,) and config.recompute_ratios == (0.25,)
    assert config.max_inflight_store_batches == 8 and config.query_score_chunk_size == 8
    for bad, match in (
        ({"typo": True}, "Unknown"),
        ({"max_apc_prefix_to_hit_ratio": -1}, "prefix"),
        ({"store_workers": 0}, "store_workers"),
        ({"selection_strategy": "unknown"}, "selection_strategy"),
        ({"selection_strategy": "sparse_q", "check_layers": [1, 2]}, "exactly one"),
        ({"selection_strategy": "sparse_q", "tail_query_tokens": 0}, "tail_query_tokens"),
        ({"recompute_ratios": [0.1, 0.2], "check_layers": [1]}, "one value"),
    ):
        with pytest.raises(ValueError, match=match):
            CacheBlendConfig.from_extra_config(bad)


def test_config_field_set_is_the_reference_set():
    names = {f for f in CacheBlendConfig.__dataclass_fields__}
    assert names == {
        "chunk_size", "local_cpu_gb", "min_retrieve_tokens", "min_hit_ratio", "min_saved_tokens",
        "max_apc_prefix_to_hit_ratio", "check_layers", "recompute_ratios", "selection_strategy",
        "query_score_chunk_size", "overflow_blocks", "tail_query_tokens", "save_decode_cache",
        "tp_global_selection", "event_pipeline", "fused_segment_copy", "cache_attention_mask",
        "lookup_timeout_ms", "store_workers", "max_inflight_store_batches",
        "strict_version_check", "ipc_root", "model_scope",
    }


def _segment(source, target, length=4):
    return BlendSegment(SegmentId("model", source + 7, source, length), target)


def test_plan_round_trip_gate_and_overlap():
    # reference tests/test_types.py:10-25
    plan = BlendPlan.from_segments(4, [_segment(0, 4), _segment(8, 12)])
    assert (plan.allocation_end, plan.hit_tokens, plan.gap_tokens) == (16, 8, 4)
    assert BlendPlan.from_dict(plan.to_dict()) == plan
    assert plan.passes_gate(4, 0.5, 0) and not plan.passes_gate(4, 0.75, 0)
    assert not plan.passes_gate(4, 0.5, 9) and not plan.passes_gate(4, 0.5, 0, 0.49)
    assert plan.passes_gate(4, 0.5, 0, 0.5)
    with pytest.raises(ValueError, match="overlap"):
        BlendPlan(0, 8, 8, (_segment(0, 0), _segment(4, 2)))
    assert plan.token_segment_map().tolist() == [-1] * 4 + [0] * 4 + [-1] * 4 + [1] * 4
    assert plan.gap_mask().tolist() == [False] * 4 + [False] * 4 + [True] * 4 + [False] * 4
    old, new = plan.hit_positions()
    assert old.tolist() == [0, 1, 2, 3, 8, 9, 10, 11] and new.tolist() == [4, 5, 6, 7, 12, 13, 14, 15]


def test_window_hashes_equal_direct_hash():
    # reference tests/test_matcher.py:6-31 (rolling == direct at every offset)
    rng = np.random.default_rng(0)
    tokens = rng.integers(0, 151_000, size=700)
    hashes = window_hashes(tokens, 256)
    for start in (0, 1, 17, 255, 444):
        assert int(hashes[start]) == content_hash(tokens[start : start + 256])
    assert window_hashes(tokens[:10], 256).shape == (0,)


def test_store_replays_reference_sequence(store_sequence):
    store = LocalPinnedCPUStore(store_sequence["chunk"], store_sequence["max_bytes"], pin_memory=False)
    known: list[tuple[SegmentId, list[int]]] = []
    for step, record in enumerate(store_sequence["log"]):
        op = record["op"]
        if op == "begin":
            sid = store.begin_put("m", record["source"], record["tokens"], 2)
            if all(entry[0] != sid for entry in known):
                known.append((sid, record["tokens"]))
        else:
            sid, tokens = known[record["index"]]
            ids = [entry[0] for entry in known]
            if op == "put":
                result = store.put_layer_host(sid, record["layer"], torch.zeros(2, 4, record["width"]))
                assert result == record["result"], step
            elif op == "reserve":
                assert store.reserve_layer(sid, record["layer"]) == record["result"], step
            elif op == "cancel":
                store.cancel_layer(sid, record["layer"])
            elif op == "abort":
                store.abort_put(sid)
            elif op == "pin":
                segs = [BlendSegment(known[j][0], 0) for j in record["indices"]]
                got = [ids.index(s.segment_id) for s in store.pin(record["request"], segs)]
                assert got == record["result"], step
            elif op == "release":
                store.release(record["request"])
            else:
                got = [ids.index(s.segment_id) for s in store.match("m", tokens, 0)]
                assert got == record["result"], step
        ids = [entry[0] for entry in known]
        assert store.current_bytes == record["bytes"], step
        assert store.committed_entries == record["committed"], step
        assert [ids.index(s) for s in store.entry_order()] == record["order"], step


def test_store_known_answers():
    # reference tests/test_storage.py:15-82
    per_entry = 2 * 2 * 4 * 2 * 4
    store = LocalPinnedCPUStore(4, max_bytes=per_entry, pin_memory=False)
    tokens1 = [10, 11, 12, 13]
    s1 = store.begin_put("m", 0, tokens1, num_layers=2)
    assert not store.put_layer(s1, 0, torch.full((2, 4, 2), 1.0))
    assert store.match("m", tokens1, 0) == ()
    assert store.put_layer(s1, 1, torch.full((2, 4, 2), 2.0))
    seg1 = store.match("m", tokens1, 0)[0]
    store.pin("r", [seg1])
    s2 = store.begin_put("m", 4, [20, 21, 22, 23], num_layers=2)
    assert store.put_layer(s2, 0, torch.full((2, 4, 2), 2.0)) is None
    assert store.current_bytes == per_entry
    store.release("r")
    tiny = LocalPinnedCPUStore(4, max_bytes=32, pin_memory=False)
    s3 = tiny.begin_put("m", 0, [1, 2, 3, 4], num_layers=1)
    assert tiny.put_layer_host(s3, 0, torch.ones(2, 4, 2)) is None
    assert tiny.current_bytes == 0 and tiny.committed_entries == 0
    view_store = LocalPinnedCPUStore(4, max_bytes=4096, pin_memory=False)
    s4 = view_store.begin_put("m", 0, [1, 2, 3, 4], num_layers=1)
    assert view_store.reserve_layer(s4, 0) and not view_store.reserve_layer(s4, 0)
    host = torch.ones(2, 8, 2)[:, 2:6]
    assert view_store.put_layer_host(s4, 0, host)
    seg = view_store.match("m", [1, 2, 3, 4], 0)[0]
    view_store.pin("r", [seg])
    assert view_store.get_layer("r", seg, 0) is host


@pytest.mark.parametrize(
    "active,gaps,base,ratio",
    [(4, 2, 2, 0.5), (4, 1, 2, 0.5), (10, 10, 10, 0.3), (10, 0, 10, 0.3), (1000, 300, 350, 0.15),
     (7, 2, 3, 0.0), (7, 2, 3, 1.0)],
)
def test_budget_matches_oracle(active, gaps, base, ratio):
    assert recompute_budget(active, gaps, base, ratio) == oracle.recompute_budget(active, gaps, base, ratio)


@pytest.mark.parametrize("radius_blocks,tail", [(0, 8), (1, 8), (3, 2), (1, 0)])
def test_sparse_q_masks_match_oracle(radius_blocks, tail):
    rng = np.random.default_rng(radius_blocks + tail)
    for gap_rate in (0.0, 0.02, 0.3):
        gaps = rng.random(300) < gap_rate
        got = sparse_q_masks(gaps, 16, radius_blocks, tail)
        want = oracle.sparse_q_masks(gaps, 16, radius_blocks, tail)
        assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
        assert got[2] == want[2]


def test_batched_reserve_and_publish_match_single_calls():
    """reserve_layers / put_layers_host == the single-chunk calls in order (one lock)."""
    import torch

    from cacheblend_b200.storage import LocalPinnedCPUStore

    def run(batched: bool):
        store = LocalPinnedCPUStore(4, 3 * 2 * 2 * 4 * 4, pin_memory=False)  # room for ~3 chunk-layers of 2 layers
        ids = [store.begin_put("m", 4 * i, [10 * i + j for j in range(4)], 2) for i in range(5)]
        log = []
        for layer in range(2):
            ok = store.reserve_layers(ids, layer) if batched else [store.reserve_layer(s, layer) for s in ids]
            log.append(ok)
            views = [torch.full((2, 4, 2), float(layer * 10 + i)) for i in range(5)]
            picked = [s for s, o in zip(ids, ok) if o]
            tensors = [v for v, o in zip(views, ok) if o]
            res = (store.put_layers_host(picked, layer, tensors) if batched
                   else [store.put_layer_host(s, layer, t) for s, t in zip(picked, tensors)])
            log.append(res)
        return log, store.entry_order(), store.current_bytes, store.committed_entries

    assert run(True) == run(False)


def test_fingerprints_match_reference_vectors():
    """The reference's own hashing.rolling_hash_values / content_hash outputs (hashes.npz):
    the O(N) window hashes, the per-chunk vectorised hashes and the scalar form agree."""
    from cacheblend_b200.matcher import TokenRangeMatcher, chunk_hashes

    gold = np.load(Path(__file__).resolve().parent / "golden" / "hashes.npz")
    tokens = gold["tokens"]
    assert np.array_equal(window_hashes(tokens, 256), gold["windows"])
    assert np.array_equal(chunk_hashes(tokens.reshape(16, 256)), gold["chunks"])
    assert [content_hash([7]), content_hash([-1, 0, 1]), content_hash([])] == gold["small"].tolist()
    records = TokenRangeMatcher(256).make_records("m", 0, tokens.tolist(), 16)
    assert [r.segment_id.content_hash for r in records] == gold["chunks"].tolist()


def test_select_tokens_routes_tp_reduction_through_the_peer_exchange():
    """With a peer exchange the TP reduction happens inside its select kernel: no
    all-reduce call, the partial scores and the reference budget go to the exchange."""
    from cacheblend_b200.selection import select_tokens

    class NoAllReduce:
        world_size = 2

        def all_reduce(self, tensor):
            raise AssertionError("the NCCL all-reduce must not run beside the peer exchange")

    class Exchange:
        def select(self, scores, base, k, capacity):
            self.args = (scores, base, k, capacity)
            return torch.arange(capacity)

    gaps = np.zeros(100, dtype=bool)
    gaps[:10] = True
    partial = torch.rand(100)
    exchange = Exchange()
    out = select_tokens(partial, gaps, 0.2, tp_group=NoAllReduce(), peer_exchange=exchange,
                        base_mask_device=torch.from_numpy(gaps.astype(np.uint8)))
    scores, base, k, capacity = exchange.args
    assert scores is partial and k == recompute_budget(100, 10, 10, 0.2) == 18 and capacity == 28
    assert out.numel() == 28


def test_executor_peer_exchange_decision(monkeypatch):
    """The executor's TP selection uses the peer exchange only with global selection,
    2-8 ranks, CUDA scores and at most MAX_TOKENS tokens; it creates the exchange once,
    and after a collective setup failure it stays on the all-reduce for good."""
    from cacheblend_b200 import executor as ex
    from cacheblend_b200.peer_exchange import MAX_TOKENS, PeerExchangeUnavailable

    made = []

    class FakeExchange:
        def __init__(self, group, max_tokens, device):
            made.append((group, max_tokens, device))

    class Group:
        def __init__(self, world):
            self.world_size = world

    def runner(world, global_selection=True):
        obj = object.__new__(ex.Qwen3BlendExecutor)
        obj.config = CacheBlendConfig(tp_global_selection=global_selection)
        obj.tp_group = Group(world)
        obj._peer = None
        obj._peer_unavailable = False
        return obj

    cuda = torch.device("cuda", 0)
    monkeypatch.setattr(ex, "PeerScoreExchange", FakeExchange)
    one = runner(2)
    first = one._peer_exchange(1000, cuda)
    assert isinstance(first, FakeExchange) and one._peer_exchange(5000, cuda) is first
    assert made == [(one.tp_group, MAX_TOKENS, cuda)]
    assert runner(1)._peer_exchange(1000, cuda) is None                      # no TP
    assert runner(16)._peer_exchange(1000, cuda) is None                     # more ranks than flags
    assert runner(2, global_selection=False)._peer_exchange(1000, cuda) is None
    assert runner(2)._peer_exchange(MAX_TOKENS + 1, cuda) is None            # too many tokens
    assert runner(2)._peer_exchange(1000, torch.device("cpu")) is None

    def unavailable(group, max_tokens, device):
        raise PeerExchangeUnavailable("rank 1 mapping rank 0: peer access unsupported")

    monkeypatch.setattr(ex, "PeerScoreExchange", unavailable)
    two = runner(2)
    assert two._peer_exchange(1000, cuda) is None and two._peer_unavailable
    monkeypatch.setattr(ex, "PeerScoreExchange", FakeExchange)
    assert two._peer_exchange(1000, cuda) is None  # no second attempt


def test_attention_modes_and_no_cpu_fallback():
    """blend_attention's exact_rounding maps onto the ABI's mode codes (reference order 1,
    flash order 2, fp32 logits 0), rejects other values, and refuses CPU tensors."""
    from cacheblend_b200.attention import _MODES, blend_attention

    assert _MODES[True] == _MODES["reference"] == 1
    assert _MODES["flash"] == 2
    assert _MODES[False] == _MODES["fused"] == 0
    q = torch.zeros(4, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        blend_attention(q, q, q, torch.arange(4), 1.0, exact_rounding="exact")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        blend_attention(q, q, q, torch.arange(4), 1.0)
