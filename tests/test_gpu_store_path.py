"""Store path on the GPU through the connector's worker API: save_kv_layer
per layer -> chunk-major gather + D2H on the Store stream -> publication into
the pinned LRU.  Published chunks must be byte-identical to the oracle's
gather of the saved slots; a later request that reuses the chunks at another
position must load (H2D + relocation) exactly what the oracle's blend load
computes from them; capacity pressure must fail closed."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200 import registry
from cacheblend_b200.config import CacheBlendConfig
from cacheblend_b200.loader import PagedBlendLoader
from cacheblend_b200.storage import LocalPinnedCPUStore
from cacheblend_b200.store_path import StorePipeline
from cacheblend_b200.types import BlendPlan

connector_module = pytest.importorskip("cacheblend_b200.connector")
from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole  # noqa: E402

pytestmark = pytest.mark.gpu

CHUNK, BS, HEADS, HD, POOL, LAYERS = 256, 16, 8, 128, 256, 3


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _pages(rng, device, layout):
    layers, planes = [], []
    for _ in range(LAYERS):
        kv = rng.integers(0, 1 << 16, size=(2, POOL, BS, HEADS, HD), dtype=np.uint16) & 0xBFFF
        planes.append(kv)
        t = torch.from_numpy(kv.view(np.int16)).view(torch.bfloat16).to(device)
        if layout == "flash_attn":
            layers.append(t)
        elif layout == "flashinfer":
            layers.append(t.permute(1, 0, 2, 3, 4).contiguous())
        else:
            layers.append((t[0].clone(), t[1].clone()))
    return layers, planes


def _worker(device, max_bytes, kv_caches, arena=False):
    connector = object.__new__(connector_module.CacheBlendConnectorV1)
    connector.config = CacheBlendConfig.from_extra_config(
        {"chunk_size": CHUNK, "strict_version_check": False, "local_cpu_gb": max_bytes / (1 << 30)}
    )
    connector.block_size = BS
    connector.engine_id = "store-test"
    connector.model_scope = "model"
    connector.tp_size = 1
    connector._role = KVConnectorRole.WORKER
    connector._init_state(KVConnectorRole.WORKER)
    connector._kv_caches = kv_caches
    connector._layer_ids = {f"model.layers.{i}.self_attn.attn": i for i in range(LAYERS)}
    connector._store = LocalPinnedCPUStore(CHUNK, max_bytes)
    if arena:  # as register_kv_caches does: one pinned arena sized by local_cpu_gb
        connector._store.attach_arena(connector._make_arena())
    connector._pipeline = StorePipeline(connector._store, BS, CHUNK, device=device)
    return connector


def _save(connector, request_id, tokens, slots, save_end):
    meta = connector_module.CacheBlendConnectorMetadata()
    meta.requests.append(connector_module.RequestMetadata(
        request_id, tokens, slots, None, True, save_end))
    connector.bind_connector_metadata(meta)
    for name, layer in connector._layer_ids.items():
        connector.save_kv_layer(name, connector._kv_caches[layer], None)
    connector.wait_for_save()


@pytest.mark.parametrize("arena", [False, True])
@pytest.mark.parametrize("layout", ["flash_attn", "flashinfer", "separate"])
def test_saved_chunks_match_oracle_gather(cuda, layout, arena):
    rng = np.random.default_rng(11)
    kv_caches, planes = _pages(rng, cuda, layout)
    connector = _worker(cuda, 1 << 30, kv_caches, arena)
    tokens = rng.integers(0, 150_000, size=3 * CHUNK + 37).tolist()
    blocks = rng.permutation(POOL)[: (len(tokens) + BS - 1) // BS]
    slots = connector_module._slot_mapping(blocks.tolist(), BS, len(tokens))
    try:
        _save(connector, "a", tokens, slots, len(tokens))
        store = connector._store
        assert store.committed_entries == 3
        segments = store.match("model", tokens, 0)
        assert [seg.target_start for seg in segments] == [0, CHUNK, 2 * CHUNK]
        store.pin("check", segments)
        for seg in segments:
            chunk_slots = slots[seg.target_start : seg.target_start + CHUNK].numpy()
            for layer in range(LAYERS):
                got = store.get_layer("check", seg, layer)
                assert got.is_pinned() and got.is_contiguous()
                want = oracle.paged_gather(planes[layer][0], planes[layer][1], chunk_slots, BS)
                assert np.array_equal(_bits(got), want), (seg.target_start, layer)
        # the partial tail chunk is never published, and a repeated save adds nothing
        _save(connector, "a2", tokens, slots, len(tokens))
        assert store.committed_entries == 3
    finally:
        connector.close()


@pytest.mark.parametrize("arena", [False, True])
def test_store_capacity_fails_closed(cuda, arena):
    rng = np.random.default_rng(12)
    kv_caches, planes = _pages(rng, cuda, "flash_attn")
    chunk_bytes = 2 * CHUNK * HEADS * HD * 2
    connector = _worker(cuda, 2 * LAYERS * chunk_bytes, kv_caches, arena)  # room for two chunks
    tokens = rng.integers(0, 150_000, size=3 * CHUNK).tolist()
    blocks = rng.permutation(POOL)[: 3 * CHUNK // BS]
    slots = connector_module._slot_mapping(blocks.tolist(), BS, len(tokens))
    try:
        _save(connector, "a", tokens, slots, len(tokens))
        store = connector._store
        assert store.current_bytes <= 2 * LAYERS * chunk_bytes
        assert store.committed_entries == 2
        if arena:
            assert store.arena.pinned_bytes <= 2 * LAYERS * chunk_bytes
        segments = store.match("model", tokens, 0)
        store.pin("check", segments)
        for seg in segments:
            chunk_slots = slots[seg.target_start : seg.target_start + CHUNK].numpy()
            for layer in range(LAYERS):
                want = oracle.paged_gather(planes[layer][0], planes[layer][1], chunk_slots, BS)
                assert np.array_equal(_bits(store.get_layer("check", seg, layer)), want)
    finally:
        connector.close()


class _Rope:
    def __init__(self, cos_sin: np.ndarray, device):
        self.head_size = HD
        self.rotary_dim = cos_sin.shape[1]
        self.is_neox_style = True
        self.cos_sin_cache = torch.from_numpy(cos_sin).to(device)


def test_saved_chunks_reload_at_new_positions(cuda):
    """Save request A, look its middle chunk up for request B at another offset, load."""
    rng = np.random.default_rng(13)
    kv_caches, planes = _pages(rng, cuda, "flash_attn")
    connector = _worker(cuda, 1 << 30, kv_caches)
    registry.register_store("store-test", 0, connector._store)
    tokens_a = rng.integers(0, 150_000, size=3 * CHUNK).tolist()
    blocks = rng.permutation(POOL)
    slots_a = connector_module._slot_mapping(blocks[:48].tolist(), BS, len(tokens_a))
    try:
        _save(connector, "a", tokens_a, slots_a, len(tokens_a))
        prefix = rng.integers(0, 150_000, size=100).tolist()
        tokens_b = prefix + tokens_a[CHUNK : 2 * CHUNK] + rng.integers(0, 150_000, size=60).tolist()
        lookup = connector_module.LocalStoreLookup("store-test")
        found = lookup.lookup_and_prefetch("b", "model", tokens_b[:-1], 0)
        assert [(seg.segment_id.source_start, seg.target_start) for seg in found] == [(CHUNK, 100)]
        plan = BlendPlan.from_segments(0, found)
        slots_b = connector_module._slot_mapping(blocks[100:130].tolist(), BS, len(tokens_b))
        max_pos = 4096
        inv = 1.0 / (1e6 ** (np.arange(0, HD, 2, dtype=np.float64) / HD))
        freqs = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
        cos_sin = np.concatenate((np.cos(freqs), np.sin(freqs)), axis=-1).astype(np.float32)
        loader = PagedBlendLoader(kv_caches, connector._store, "b", plan, slots_b, BS, connector.config,
                                  load_stream=torch.cuda.Stream(cuda))
        rope = _Rope(cos_sin, cuda)
        table = oracle.f32_to_bf16(cos_sin)
        loader.prefetch(0, rope)
        saved_slots = slots_a[CHUNK : 2 * CHUNK].numpy()
        for layer in range(LAYERS):
            staging = _bits(loader.get(layer))
            if layer + 1 < LAYERS:
                loader.prefetch(layer + 1, rope)
            host = oracle.paged_gather(planes[layer][0], planes[layer][1], saved_slots, BS)
            want = oracle.blend_load(
                oracle.BF16, plan.allocation_end, 0, planes[layer][0], planes[layer][1],
                slots_b[: plan.allocation_end].numpy(), BS, [(CHUNK, 100, CHUNK, host)],
                np.ones(1, dtype=np.int32), table, HD, HD, True,
            )
            assert np.array_equal(staging, want), layer
        lookup.cancel("b")
    finally:
        registry.unregister_store("store-test", 0)
        connector.close()


def test_arena_fragmented_slots_match_oracle(cuda):
    """Eviction leaves the arena's free slots scattered: a later batch lands in
    runs of consecutive slots (one strided copy each) and single slots, and every
    published chunk still equals the oracle's gather; pinned memory never grows."""
    rng = np.random.default_rng(21)
    kv_caches, planes = _pages(rng, cuda, "flash_attn")
    chunk_bytes = 2 * CHUNK * HEADS * HD * 2
    connector = _worker(cuda, 6 * LAYERS * chunk_bytes, kv_caches, arena=True)  # six entries
    store = connector._store
    try:
        requests = {}
        for name in ("a", "b", "c"):
            tokens = rng.integers(0, 150_000, size=3 * CHUNK).tolist()
            blocks = rng.permutation(POOL)[: 3 * CHUNK // BS]
            slots = connector_module._slot_mapping(blocks.tolist(), BS, len(tokens))
            requests[name] = (tokens, slots)
            if name == "c":
                # keep a's middle chunk and b's last chunk pinned: c must take slots
                # 0, 2 and 3 (a's first and last, b's first) around them
                seg_a = store.match("model", requests["a"][0], 0)
                seg_b = store.match("model", requests["b"][0], 0)
                store.pin("keep", (seg_a[1], seg_b[2]))
            _save(connector, name, tokens, slots, len(tokens))
        assert store.arena.used_slots == 6 and store.arena.pinned_bytes == 6 * LAYERS * chunk_bytes
        slot_of = {sid: entry.slot for sid, entry in store._entries.items()}
        tokens, slots = requests["c"]
        segments = store.match("model", tokens, 0)
        assert len(segments) == 3
        assert sorted(slot_of[seg.segment_id] for seg in segments) == [0, 2, 3]
        store.pin("check", segments)
        for seg in segments:
            chunk_slots = slots[seg.target_start : seg.target_start + CHUNK].numpy()
            for layer in range(LAYERS):
                want = oracle.paged_gather(planes[layer][0], planes[layer][1], chunk_slots, BS)
                assert np.array_equal(_bits(store.get_layer("check", seg, layer)), want)
        # the pinned survivors are intact too
        for name, index in (("a", 1), ("b", 2)):
            tok, sl = requests[name]
            seg = store.match("model", tok, 0)
            assert len(seg) >= 1
            seg = [x for x in seg if x.target_start == index * CHUNK][0]
            store.pin("old", [seg])
            chunk_slots = sl[seg.target_start : seg.target_start + CHUNK].numpy()
            for layer in range(LAYERS):
                want = oracle.paged_gather(planes[layer][0], planes[layer][1], chunk_slots, BS)
                assert np.array_equal(_bits(store.get_layer("old", seg, layer)), want)
    finally:
        connector.close()



def test_arena_reservation_precedes_the_gather(cuda):
    """A batch whose chunks all fail closed at the arena reservation launches no
    gather and copies nothing; an enqueue that raises after its slot was reserved
    gives the slot and the entry's layer reservation back."""
    rng = np.random.default_rng(14)
    kv_caches, _ = _pages(rng, cuda, "flash_attn")
    chunk_bytes = 2 * CHUNK * HEADS * HD * 2
    connector = _worker(cuda, 2 * LAYERS * chunk_bytes, kv_caches, arena=True)  # two entries
    pipe, store = connector._pipeline, connector._store
    tokens = rng.integers(0, 150_000, size=4 * CHUNK).tolist()
    blocks = rng.permutation(POOL)[: 4 * CHUNK // BS]
    slots = connector_module._slot_mapping(blocks.tolist(), BS, len(tokens))
    try:
        _save(connector, "a", tokens[: 2 * CHUNK], slots[: 2 * CHUNK], 2 * CHUNK)
        store.pin("keep", store.match("model", tokens[: 2 * CHUNK], 0))
        pipe.kernel_events, before = [], pipe.d2h_bytes
        _save(connector, "b", tokens[2 * CHUNK :], slots[2 * CHUNK :], 2 * CHUNK)
        assert pipe.kernel_events == [] and pipe.d2h_bytes == before
        assert store.committed_entries == 2 and store.arena.used_slots == 2
        store.release("keep")
        sids = store.begin_put_chunks("model", 0, tokens[2 * CHUNK :], 1, LAYERS)
        assert store.reserve_layers(sids, 0) == [True]
        bad = torch.full((CHUNK,), POOL * BS, dtype=torch.long)  # one past the last page slot
        with pytest.raises(IndexError):  # host-side range check, after the slot reservation
            pipe.enqueue([(sids[0], 0, CHUNK)], kv_caches[0], bad, "c")
        assert sids[0] not in store._entries
        assert store.committed_entries == 1 and store.arena.used_slots == 1  # one evicted for it
        assert pipe.kernel_events == []
    finally:
        connector.close()
