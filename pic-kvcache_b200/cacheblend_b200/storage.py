"""Per-rank pinned-CPU LRU store: the Store path's publication target.

Entry lifecycle and eviction are the contract of LocalPinnedCPUStore
(cacheblend_vllm/storage.py:35-294), kept identical because request plans,
fail-closed capacity behaviour and hit rates depend on them:

* an entry is created by ``begin_put`` and becomes matchable ("committed")
  only when every layer has been published;
* ``put_layer_host`` stores the caller's CPU tensor (a view is kept, never
  copied) and returns True when it committed the entry, False when more
  layers are needed (or the entry was already committed), None when the
  whole entry was rejected to respect ``max_bytes`` or had failed;
* eviction walks entries from least to most recently used and removes only
  committed, unpinned entries other than the one being written;
* a failed/aborted entry is discarded as soon as no layer transfer is
  reserved and no request pins it.

The bytes of a layer are ``numel * element_size`` of the published tensor.

Arena mode (``attach_arena``, used by the Store path): an entry's layers live
in one slot of a ``PinnedArena`` taken when the entry's first layer transfer is
reserved (``arena_reserve``).  When no slot is free, committed unpinned entries
other than the writer are evicted in LRU order until one is; when none can be,
the entry fails closed exactly as an over-budget put does.  Removing an entry
returns its slot.  The byte accounting of published layers is unchanged, and
the arena's size never exceeds ``max_bytes``.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from collections.abc import Iterable, Sequence
from dataclasses import dataclass, field

import torch

from .matcher import FingerprintRecord, TokenRangeMatcher
from .types import BlendSegment, SegmentId


@dataclass(slots=True)
class _Entry:
    record: FingerprintRecord
    num_layers: int
    layers: dict[int, torch.Tensor] = field(default_factory=dict)
    reserved_layers: set[int] = field(default_factory=set)
    size_bytes: int = 0
    pin_count: int = 0
    committed: bool = False
    failed: bool = False
    last_access: float = field(default_factory=time.monotonic)
    slot: int | None = None  # arena slot holding every layer (arena mode)

    def idle(self) -> bool:
        return not self.reserved_layers and not self.pin_count


def _nbytes(tensor: torch.Tensor) -> int:
    return tensor.numel() * tensor.element_size()


class LocalPinnedCPUStore:
    def __init__(self, chunk_size: int, max_bytes: int, pin_memory: bool = True):
        if max_bytes <= 0:
            raise ValueError("max_bytes must be positive")
        self.matcher = TokenRangeMatcher(chunk_size)
        self.max_bytes = int(max_bytes)
        self.pin_memory = pin_memory
        self._entries: OrderedDict[SegmentId, _Entry] = OrderedDict()
        # the committed entries in the same least-to-most recent order: the
        # eviction walk visits only these, so writers under capacity pressure
        # do not rescan every in-flight entry on each publication
        self._committed: OrderedDict[SegmentId, _Entry] = OrderedDict()
        self._bytes = 0
        # per request, its pinned segment ids in pin order (a dict: O(1) membership for the
        # loader's per-layer lookups, insertion order for release)
        self._request_pins: dict[str, dict[SegmentId, None]] = {}
        self._lock = threading.RLock()
        self.arena = None  # PinnedArena once attached

    # ---- introspection ------------------------------------------------------
    @property
    def current_bytes(self) -> int:
        with self._lock:
            return self._bytes

    @property
    def committed_entries(self) -> int:
        return len(self.matcher)

    def entry_order(self) -> list[SegmentId]:
        """Entries from least to most recently used (for tests and tooling)."""
        with self._lock:
            return list(self._entries)

    # ---- arena mode ------------------------------------------------------------
    def attach_arena(self, arena) -> None:
        """Publish the Store path's layers into ``arena`` slots from now on."""
        with self._lock:
            if self.arena is not None and self.arena is not arena:
                raise RuntimeError("the store already has an arena")
            self.arena = arena

    def arena_reserve(self, segment_ids: Sequence[SegmentId], layer_id: int) -> list[int | None]:
        """Per segment, the arena slot that layer ``layer_id`` is to be copied into, or
        None when the transfer is dropped (unknown, failed or committed entry, or no slot
        could be freed: the entry then fails closed and its reservation is released)."""
        if self.arena is None:
            raise RuntimeError("no arena attached")
        out: list[int | None] = []
        with self._lock:
            for sid in segment_ids:
                entry = self._entries.get(sid)
                if entry is None:
                    out.append(None)
                    continue
                self._check_layer(entry, layer_id)
                if entry.committed or entry.failed:
                    entry.reserved_layers.discard(layer_id)
                    if entry.failed and entry.idle():
                        self._remove(sid, entry)
                    out.append(None)
                    continue
                if entry.slot is None:
                    slot = self.arena.alloc()
                    if slot is None:
                        self._evict_slot(exclude=sid)
                        slot = self.arena.alloc()
                    if slot is None:
                        entry.reserved_layers.discard(layer_id)
                        entry.failed = True
                        if entry.idle():
                            self._remove(sid, entry)
                        out.append(None)
                        continue
                    entry.slot = slot
                out.append(entry.slot)
        return out

    def _evict_slot(self, exclude: SegmentId | None = None) -> None:
        """Evict the least recently used committed, unpinned entry holding a slot."""
        for sid, entry in self._committed.items():
            if sid == exclude or entry.pin_count or entry.slot is None:
                continue
            self._remove(sid, entry)
            return

    # ---- writers -------------------------------------------------------------
    def begin_put(
        self, model_scope: str, source_start: int, tokens: Sequence[int], num_layers: int
    ) -> SegmentId:
        if num_layers <= 0:
            raise ValueError("num_layers must be positive")
        record = self.matcher.make_record(model_scope, source_start, tokens)
        with self._lock:
            return self._begin(record, num_layers)

    def begin_put_chunks(
        self, model_scope: str, first_start: int, tokens: Sequence[int], count: int, num_layers: int
    ) -> list[SegmentId]:
        """``begin_put`` of ``count`` consecutive chunks of ``tokens`` from ``first_start``,
        fingerprinted in one vectorised pass; same ids, entries and LRU order as the
        equivalent sequence of ``begin_put`` calls."""
        if num_layers <= 0:
            raise ValueError("num_layers must be positive")
        records = self.matcher.make_records(model_scope, first_start, tokens, count)
        with self._lock:
            return [self._begin(record, num_layers) for record in records]

    def _begin(self, record: FingerprintRecord, num_layers: int) -> SegmentId:
        sid = record.segment_id
        entry = self._entries.get(sid)
        if entry is None:
            self._entries[sid] = _Entry(record=record, num_layers=num_layers)
            return sid
        if entry.record.tokens != record.tokens:
            raise RuntimeError("content-hash collision for an existing segment id")
        if entry.num_layers != num_layers:
            raise ValueError("num_layers changed for an existing segment")
        self._touch(sid, entry)
        return sid

    def put_layer(self, segment_id: SegmentId, layer_id: int, kv: torch.Tensor) -> bool | None:
        """Copy ``kv`` to host memory and publish it (see put_layer_host)."""
        with self._lock:
            entry = self._entries.get(segment_id)
            if entry is None:
                raise KeyError(segment_id)
            self._check_layer(entry, layer_id)
        host = kv.detach().to(device="cpu", copy=True).contiguous()
        if self.pin_memory and not host.is_pinned():
            try:
                host = host.pin_memory()
            except RuntimeError:
                pass  # hosts without a pinning allocator: correctness does not depend on it
        return self.put_layer_host(segment_id, layer_id, host)

    def reserve_layer(self, segment_id: SegmentId, layer_id: int) -> bool:
        """Claim one layer for an asynchronous transfer; False if already present/claimed."""
        with self._lock:
            return self._reserve(segment_id, layer_id)

    def reserve_layers(self, segment_ids: Sequence[SegmentId], layer_id: int) -> list[bool]:
        """``reserve_layer`` for each segment in order, under one lock acquisition."""
        with self._lock:
            return [self._reserve(sid, layer_id) for sid in segment_ids]

    def _reserve(self, segment_id: SegmentId, layer_id: int) -> bool:
        entry = self._entries.get(segment_id)
        if entry is None:
            return False
        self._check_layer(entry, layer_id)
        if entry.failed or layer_id in entry.layers or layer_id in entry.reserved_layers:
            return False
        entry.reserved_layers.add(layer_id)
        return True

    def cancel_layer(self, segment_id: SegmentId, layer_id: int) -> None:
        with self._lock:
            entry = self._entries.get(segment_id)
            if entry is None:
                return
            entry.reserved_layers.discard(layer_id)
            if not entry.committed:
                entry.failed = True
            if entry.failed and entry.idle():
                self._remove(segment_id, entry)

    def put_layer_host(
        self, segment_id: SegmentId, layer_id: int, cpu_tensor: torch.Tensor
    ) -> bool | None:
        if cpu_tensor.device.type != "cpu":
            raise ValueError("put_layer_host requires a CPU tensor")
        with self._lock:
            return self._put_host(segment_id, layer_id, cpu_tensor, _nbytes(cpu_tensor))

    def put_layers_host(
        self, segment_ids: Sequence[SegmentId], layer_id: int, cpu_tensors: Sequence[torch.Tensor]
    ) -> list[bool | None]:
        """``put_layer_host`` for each (segment, tensor) pair in order, under one lock
        acquisition (the Store path publishes a whole batch of one layer at once)."""
        if len(segment_ids) != len(cpu_tensors):
            raise ValueError("one tensor per segment is required")
        if any(t.device.type != "cpu" for t in cpu_tensors):
            raise ValueError("put_layer_host requires a CPU tensor")
        with self._lock:
            return [self._put_host(sid, layer_id, t, _nbytes(t)) for sid, t in zip(segment_ids, cpu_tensors)]

    def _put_host(
        self, segment_id: SegmentId, layer_id: int, cpu_tensor: torch.Tensor, nbytes: int
    ) -> bool | None:
        entry = self._entries.get(segment_id)
        if entry is None:
            return None
        self._check_layer(entry, layer_id)
        if entry.failed:
            entry.reserved_layers.discard(layer_id)
            if entry.idle():
                self._remove(segment_id, entry)
            return None
        if entry.committed:
            entry.reserved_layers.discard(layer_id)
            return False  # content-addressed entries are immutable
        old = entry.layers.get(layer_id)
        old_bytes = _nbytes(old) if old is not None else 0
        growth = nbytes - old_bytes
        if growth > 0:
            self._evict(required_bytes=growth, exclude=segment_id)
        if self._bytes + growth > self.max_bytes:
            # fail closed: never expose a partial entry, never exceed the cap
            entry.reserved_layers.discard(layer_id)
            entry.failed = True
            if entry.idle():
                self._remove(segment_id, entry)
            return None
        entry.reserved_layers.discard(layer_id)
        entry.layers[layer_id] = cpu_tensor
        entry.size_bytes += growth
        self._bytes += growth
        entry.last_access = time.monotonic()
        newly_committed = not entry.committed and len(entry.layers) == entry.num_layers
        if newly_committed:
            entry.committed = True
            self.matcher.register(entry.record)
            self._committed[segment_id] = entry
        self._touch(segment_id, entry)
        return newly_committed

    def abort_put(self, segment_id: SegmentId) -> None:
        with self._lock:
            entry = self._entries.get(segment_id)
            if entry is None or entry.committed:
                return
            entry.failed = True
            if entry.idle():
                self._remove(segment_id, entry)

    # ---- readers -------------------------------------------------------------
    def match(
        self, model_scope: str, tokens: Sequence[int], start_offset: int
    ) -> tuple[BlendSegment, ...]:
        return self.validate(self.matcher.match(model_scope, tokens, start_offset))

    def validate(self, segments: Iterable[BlendSegment]) -> tuple[BlendSegment, ...]:
        kept: list[BlendSegment] = []
        with self._lock:
            for seg in segments:
                entry = self._entries.get(seg.segment_id)
                if entry is not None and entry.committed:
                    self._touch(seg.segment_id, entry)
                    kept.append(seg)
        return tuple(kept)

    def pin(self, request_id: str, segments: Iterable[BlendSegment]) -> tuple[BlendSegment, ...]:
        """Atomically pin the committed subset of ``segments`` for one request."""
        wanted = tuple(segments)
        with self._lock:
            self.release(request_id)
            kept: list[BlendSegment] = []
            for seg in wanted:
                entry = self._entries.get(seg.segment_id)
                if entry is None or not entry.committed:
                    continue
                entry.pin_count += 1
                self._touch(seg.segment_id, entry)
                kept.append(seg)
            if kept:
                self._request_pins[request_id] = dict.fromkeys(seg.segment_id for seg in kept)
            return tuple(kept)

    def release(self, request_id: str) -> None:
        with self._lock:
            for sid in self._request_pins.pop(request_id, ()):
                entry = self._entries.get(sid)
                if entry is not None:
                    entry.pin_count = max(0, entry.pin_count - 1)
            self._evict()

    def get_layer(self, request_id: str, segment: BlendSegment, layer_id: int) -> torch.Tensor:
        with self._lock:
            return self._pinned_layer(self._request_pins.get(request_id, {}), request_id, segment,
                                      layer_id)

    def get_layers(self, request_id: str, segments, layer_id: int) -> list[torch.Tensor]:
        """``get_layer`` for every segment in order, under one lock acquisition: the same
        checks, errors and LRU touches as the calls one by one (the loader's per-layer lookup)."""
        with self._lock:
            pins = self._request_pins.get(request_id, {})
            return [self._pinned_layer(pins, request_id, seg, layer_id) for seg in segments]

    def _pinned_layer(self, pins: dict, request_id: str, segment: BlendSegment,
                      layer_id: int) -> torch.Tensor:
        sid = segment.segment_id
        if sid not in pins:
            raise RuntimeError(f"segment {sid} is not pinned by {request_id}")
        entry = self._entries.get(sid)
        if entry is None or not entry.committed:
            raise KeyError(sid)
        tensor = entry.layers.get(layer_id)
        if tensor is None:
            raise KeyError(f"layer {layer_id} is not stored for {sid}")
        self._touch(sid, entry)
        return tensor

    def clear(self) -> None:
        with self._lock:
            for sid, entry in list(self._entries.items()):
                self.matcher.unregister(sid)
                if entry.slot is not None:
                    self.arena.free(entry.slot)
                    entry.slot = None
            self._entries.clear()
            self._committed.clear()
            self._request_pins.clear()
            self._bytes = 0

    # ---- internals -----------------------------------------------------------
    @staticmethod
    def _check_layer(entry: _Entry, layer_id: int) -> None:
        if not 0 <= layer_id < entry.num_layers:
            raise ValueError(f"layer {layer_id} is outside [0, {entry.num_layers})")

    def _touch(self, segment_id: SegmentId, entry: _Entry) -> None:
        entry.last_access = time.monotonic()
        self._entries.move_to_end(segment_id)
        if entry.committed:
            self._committed.move_to_end(segment_id)

    def _remove(self, segment_id: SegmentId, entry: _Entry) -> None:
        self.matcher.unregister(segment_id)
        self._entries.pop(segment_id, None)
        self._committed.pop(segment_id, None)
        self._bytes -= entry.size_bytes
        if entry.slot is not None:
            # later copies into the slot are ordered after any still in flight
            # (one Store stream), and readers pin the entries they read
            self.arena.free(entry.slot)
            entry.slot = None

    def _evict(self, required_bytes: int = 0, exclude: SegmentId | None = None) -> None:
        if self._bytes + required_bytes <= self.max_bytes:
            return
        freed = 0
        victims: list[tuple[SegmentId, _Entry]] = []
        for sid, entry in self._committed.items():
            if self._bytes - freed + required_bytes <= self.max_bytes:
                break
            if sid == exclude or entry.pin_count:
                continue
            victims.append((sid, entry))
            freed += entry.size_bytes
        for sid, entry in victims:
            self._remove(sid, entry)
