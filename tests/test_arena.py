"""Pinned arena of the Store path and the store's arena mode, on CPU (plain host
memory stands in for pinned memory): slot allocation order, growth by
segments up to the byte budget, slot reuse after eviction, fail-closed
reservation, and slots returned on abort / clear."""

from __future__ import annotations

import pytest
import torch

from cacheblend_b200.arena import PinnedArena
from cacheblend_b200.storage import LocalPinnedCPUStore

LAYER_SHAPE = (2, 4, 2, 4)  # [K/V, chunk, heads, head] of one layer of one chunk
LAYER_BYTES = 2 * 4 * 2 * 4 * 4  # fp32
LAYERS = 3


def _arena(entries, segment_entries=2):
    entry = LAYER_BYTES * LAYERS
    return PinnedArena(LAYER_BYTES, LAYERS, entries * entry, segment_bytes=segment_entries * entry,
                       pin_memory=False)


def test_arena_next_fit_and_growth():
    arena = _arena(5)
    assert arena.capacity == 5 and arena.pinned_bytes == 0
    got = [arena.alloc() for _ in range(5)]
    assert got == [0, 1, 2, 3, 4]
    assert arena.pinned_bytes == 5 * LAYER_BYTES * LAYERS  # three segments: 2 + 2 + 1 entries
    assert arena.alloc() is None
    arena.free(1)
    arena.free(2)
    assert arena.alloc() == 1 and arena.alloc() == 2  # next fit wraps to the freed run
    assert arena.pinned_bytes == 5 * LAYER_BYTES * LAYERS  # no growth past the budget
    with pytest.raises(ValueError):
        arena.free(7)


def test_arena_views_address_their_own_bytes():
    arena = _arena(4)
    slots = [arena.alloc() for _ in range(4)]
    for slot in slots:
        for layer in range(LAYERS):
            arena.layer_view(slot, layer, LAYER_SHAPE, torch.float32).fill_(slot * 10 + layer)
    for slot in slots:
        for layer in range(LAYERS):
            view = arena.layer_view(slot, layer, LAYER_SHAPE, torch.float32)
            assert torch.all(view == slot * 10 + layer)
            assert view.data_ptr() == arena.layer_ptr(slot, layer)
    # consecutive slots of one segment are one entry apart
    assert arena.layer_ptr(1, 0) - arena.layer_ptr(0, 0) == arena.entry_bytes


def _store(entries):
    store = LocalPinnedCPUStore(4, entries * LAYER_BYTES * LAYERS, pin_memory=False)
    store.attach_arena(_arena(entries))
    return store


def _publish(store, sids, slots, layer):
    views = [store.arena.layer_view(slot, layer, LAYER_SHAPE, torch.float32) for slot in slots]
    return store.put_layers_host(sids, layer, views)


def _save(store, first, count):
    tokens = list(range((first + count) * 4))  # chunk i = tokens[(first + i) * 4 : ...]
    sids = store.begin_put_chunks("m", first * 4, tokens, count, LAYERS)
    for layer in range(LAYERS):
        store.reserve_layers(sids, layer)
        slots = store.arena_reserve(sids, layer)
        kept = [(sid, slot) for sid, slot in zip(sids, slots) if slot is not None]
        if kept:
            _publish(store, [sid for sid, _ in kept], [slot for _, slot in kept], layer)
    return sids


def test_store_arena_commit_and_read_back():
    store = _store(4)
    sids = _save(store, 0, 3)
    assert store.committed_entries == 3
    assert [store._entries[sid].slot for sid in sids] == [0, 1, 2]
    segs = store.match("m", list(range(12)), 0)
    store.pin("r", segs)
    for seg in segs:
        got = store.get_layer("r", seg, 1)
        assert got.data_ptr() == store.arena.layer_ptr(store._entries[seg.segment_id].slot, 1)
    assert store.current_bytes == 3 * LAYERS * LAYER_BYTES


def test_store_arena_evicts_lru_unpinned_for_a_slot():
    store = _store(3)
    first = _save(store, 0, 3)
    segs = store.match("m", list(range(12)), 0)
    store.pin("keep", [segs[0]])  # entry 0 pinned; LRU order now 1, 2, 0
    second = _save(store, 10, 2)  # needs two slots: evicts entries 1 and 2
    assert store.committed_entries == 3
    assert first[0] in store._entries and first[1] not in store._entries and first[2] not in store._entries
    assert sorted(store._entries[sid].slot for sid in second) == [1, 2]
    assert store.arena.used_slots == 3
    assert store.arena.pinned_bytes <= store.max_bytes


def test_store_arena_fails_closed_when_everything_is_pinned():
    store = _store(2)
    _save(store, 0, 2)
    store.pin("keep", store.match("m", list(range(8)), 0))
    sids = store.begin_put_chunks("m", 40, list(range(44)), 1, LAYERS)
    store.reserve_layers(sids, 0)
    assert store.arena_reserve(sids, 0) == [None]
    assert sids[0] not in store._entries  # failed, idle -> discarded
    assert store.committed_entries == 2 and store.arena.used_slots == 2


def test_store_arena_slots_return_on_abort_and_clear():
    store = _store(3)
    sids = store.begin_put_chunks("m", 0, list(range(8)), 2, LAYERS)
    store.reserve_layers(sids, 0)
    assert store.arena_reserve(sids, 0) == [0, 1]
    store.cancel_layer(sids[0], 0)  # the transfer of entry 0 is given up: entry fails, idle
    assert store.arena.used_slots == 1
    store.abort_put(sids[1])  # failed, but its layer-0 transfer is still reserved
    assert store.arena.used_slots == 1
    assert _publish(store, [sids[1]], [1], 0) == [None]  # the late put discards it
    assert store.arena.used_slots == 0 and store.current_bytes == 0
    _save(store, 5, 3)
    assert store.arena.used_slots == 3
    store.clear()
    assert store.arena.used_slots == 0 and store.committed_entries == 0


def test_layer_views_match_layer_view_across_runs_and_segments():
    arena = _arena(7, segment_entries=3)  # segments of 3, 3 and 1 entries
    slots = [arena.alloc() for _ in range(7)]
    for slot in slots:
        for layer in range(LAYERS):
            arena.layer_view(slot, layer, LAYER_SHAPE, torch.float32).fill_(slot * 10 + layer)
    picks = [0, 1, 2, 3, 4, 6, 5, 1]  # runs inside a segment, across a boundary, out of order
    views = arena.layer_views(picks, 2, LAYER_SHAPE, torch.float32)
    assert len(views) == len(picks)
    for slot, view in zip(picks, views):
        assert view.shape == LAYER_SHAPE and view.is_contiguous()
        assert view.data_ptr() == arena.layer_ptr(slot, 2)
        assert torch.all(view == slot * 10 + 2)
    assert arena.layer_views([], 0, LAYER_SHAPE, torch.float32) == []
