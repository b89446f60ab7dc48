"""Store path: layerwise writeback of complete chunks into the pinned LRU (K5).

Same ordering and publication semantics as the reference connector's Store
stream (cacheblend_vllm/connector.py:384-549):

* ``enqueue`` (``_enqueue_store_batch``): take one of
  ``max_inflight_store_batches`` slots, make the single Store stream wait for
  the serving stream, gather the batch's paged KV into a per-request reusable
  device staging buffer, copy it to a fresh pinned host batch on the same
  stream, record an event and hand the batch to a publisher thread;
* ``_publish_after_event``: wait for the event, publish every chunk's host view
  with ``put_layer_host``; any exception aborts all of the batch's segments;
* ``wait_for_save``: synchronize the Store stream, join every publication,
  then drop the staging buffers (they may still be read until then).

B200 specifics: the staging is chunk-major ``[chunks, 2, chunk, H, D]`` so the
gather is one ``cb_paged_gather`` launch and every published chunk view is
contiguous (one DMA when the chunk is loaded again).  With a pinned arena
attached to the store, the chunks' slots are reserved before the gather (a
batch whose chunks all fail closed launches nothing) and each chunk's layer
is copied straight into its entry's arena slot: chunks in consecutive slots go
in one strided copy-engine transfer (``cb_copy_rows_d2h``, row pitch = the
entry size), so a batch of
chunks begun together is still one transfer.  Without an arena the batch goes
to a fresh pinned buffer in one transfer and its chunks are published as views.
"""

from __future__ import annotations

import math
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any

import torch

from . import _native
from .kv_layout import describe_paged, device_slots, gather_chunk_major
from .storage import LocalPinnedCPUStore
from .trace import PipelineTracer


class StorePipeline:
    """One Store stream, its staging buffers and its publisher threads."""

    def __init__(
        self,
        store: LocalPinnedCPUStore,
        block_size: int,
        chunk_size: int,
        store_workers: int = 1,
        max_inflight_store_batches: int = 8,
        tracer: PipelineTracer | None = None,
        device: torch.device | None = None,
    ):
        self.store = store
        self.block_size = block_size
        self.chunk_size = chunk_size
        self.tracer = tracer or PipelineTracer("store")
        self._slots = threading.Semaphore(max_inflight_store_batches)
        self._pool = ThreadPoolExecutor(max_workers=store_workers,
                                        thread_name_prefix="cacheblend-b200-save")
        self._lock = threading.Lock()
        self._futures: set[Future[bool]] = set()
        self._pending_counts: dict[str, int] = {}
        self._staging: dict[str, torch.Tensor] = {}
        self._retired: list[torch.Tensor] = []
        # per request: (host slots identity, device slots) -- every layer of a
        # forward stores the same slots, so they are checked and copied once
        self._slot_cache: dict[str, tuple[tuple[int, ...], torch.Tensor, torch.Tensor]] = {}
        self._layouts: dict[tuple, Any] = {}
        # when a list, (start, end, staging bytes) of every gather launch
        self.kernel_events: list | None = None
        self.d2h_bytes = 0  # bytes copied device -> host since construction
        self.stream = torch.cuda.Stream(device=device) if device is not None else torch.cuda.Stream()

    # ------------------------------------------------------------- enqueue
    def enqueue(
        self,
        pending: list[tuple[Any, int, int]],
        kv_layer: Any,
        slots: torch.Tensor,
        request_id: str,
        store_enqueued_ns: int | None = None,
    ) -> None:
        """Gather + D2H of one request's chunks of one layer on the Store stream.

        With an arena the chunks' slots are reserved first: a batch whose chunks all
        fail closed there launches nothing and takes no in-flight slot.  When the
        enqueue itself fails, the batch's layer reservations are given up
        (``cancel_layer``), so no entry or arena slot waits for a put that never comes."""
        try:
            paged = self._describe(kv_layer)
            _native.require_cuda(paged.key)
            chunks = len(pending)
            if chunks * self.chunk_size != slots.numel():
                raise ValueError("slots must cover the pending chunks exactly")
            shape = (chunks, 2, self.chunk_size, *paged.row.dims)
            arena_slots = self._arena_reserve(pending, shape, paged.dtype)
        except Exception:
            self._cancel(pending)
            raise
        if arena_slots is not None and all(slot is None for slot in arena_slots):
            with self._lock:
                self._pending_counts[request_id] = self._pending_counts.get(request_id, 0) + 1
            return
        self._slots.acquire()
        try:
            serving = torch.cuda.current_stream(paged.device)
            with torch.cuda.stream(self.stream):
                self.stream.wait_stream(serving)
                staging = self._staging.get(request_id)
                if staging is None or tuple(staging.shape) != shape:
                    if staging is not None:
                        # a later layer may store fewer chunks after a capacity
                        # rejection; keep the old buffer alive until the Store
                        # stream drains (its D2H may still read it)
                        self._retired.append(staging)
                    staging = torch.empty(shape, dtype=paged.dtype, device=paged.device)
                    self._staging[request_id] = staging
                identity = (slots.data_ptr(), slots.numel(), slots.stride(0), paged.num_blocks)
                cached = self._slot_cache.get(request_id)
                if cached is not None and cached[0] == identity and slots.device.type == "cpu":
                    device_slots_ = cached[2]
                else:
                    device_slots_ = device_slots(slots, paged, self.block_size)
                    # the host tensor is kept with its copy so that its address
                    # cannot be reused by other slots while the entry lives
                    self._slot_cache[request_id] = (identity, slots, device_slots_)
                if self.kernel_events is not None:
                    begin = torch.cuda.Event(enable_timing=True)
                    begin.record(self.stream)
                gather_chunk_major(paged, device_slots_, staging, stream=self.stream)
                if self.kernel_events is not None:
                    finish = torch.cuda.Event(enable_timing=True)
                    finish.record(self.stream)
                    self.kernel_events.append((begin, finish, staging.numel() * staging.element_size()))
                if arena_slots is not None:
                    self._arena_copy(pending, arena_slots, staging)
                    host = None
                else:
                    host = torch.empty(shape, dtype=paged.dtype, pin_memory=True)
                    host.copy_(staging, non_blocking=True)
                    self.d2h_bytes += host.numel() * host.element_size()
                event = torch.cuda.Event()
                event.record(self.stream)
                device_slots_.record_stream(self.stream)
            future = self._pool.submit(
                self._publish_after_event, event, pending, host, request_id, store_enqueued_ns,
                arena_slots, shape[1:], paged.dtype,
            )
        except Exception:
            self._slots.release()
            self._cancel(pending)
            raise
        with self._lock:
            self._futures.add(future)
            self._pending_counts[request_id] = self._pending_counts.get(request_id, 0) + 1
        future.add_done_callback(self._done)

    def _arena_reserve(self, pending: list[tuple[Any, int, int]], shape: tuple[int, ...],
                       dtype: torch.dtype) -> list | None:
        """Reserve arena slots for the batch's chunks.  Returns the slot per chunk (None:
        dropped, fail closed) or None when the batch does not use the arena (no arena,
        mixed layers or another chunk geometry)."""
        arena = self.store.arena
        if arena is None or not pending:
            return None
        layer_id = pending[0][1]
        chunk_bytes = math.prod(shape[1:]) * dtype.itemsize
        if chunk_bytes != arena.layer_bytes or any(layer != layer_id for _, layer, _ in pending):
            return None
        return self.store.arena_reserve([sid for sid, _, _ in pending], layer_id)

    def _arena_copy(self, pending: list[tuple[Any, int, int]], slots: list, staging: torch.Tensor) -> None:
        """Copy each reserved chunk's layer from the staging into its slot on the Store
        stream, one strided transfer per run of consecutive slots."""
        arena = self.store.arena
        layer_id = pending[0][1]
        chunk_bytes = staging[0].numel() * staging.element_size()
        kept = [(i, slot) for i, slot in enumerate(slots) if slot is not None]
        stream = self.stream.cuda_stream
        start = 0
        while start < len(kept):
            end = start + 1
            while (end < len(kept) and kept[end][0] == kept[end - 1][0] + 1
                   and kept[end][1] == kept[end - 1][1] + 1
                   and kept[end][1] // arena.slots_per_segment == kept[start][1] // arena.slots_per_segment):
                end += 1
            index, slot = kept[start]
            _native.call("cb_copy_rows_d2h", arena.layer_ptr(slot, layer_id), arena.entry_bytes,
                         staging[index].data_ptr(), chunk_bytes, chunk_bytes, end - start, stream)
            self.d2h_bytes += (end - start) * chunk_bytes
            start = end

    def _cancel(self, pending: list[tuple[Any, int, int]]) -> None:
        for segment_id, layer_id, _ in pending:
            self.store.cancel_layer(segment_id, layer_id)

    def _describe(self, kv_layer: Any):
        """``describe_paged`` memoised on the layer tensors' identity and geometry."""
        tensors = (kv_layer,) if isinstance(kv_layer, torch.Tensor) else tuple(kv_layer)
        key = tuple((t.data_ptr(), tuple(t.shape), t.stride(), t.dtype, t.device) for t in tensors)
        paged = self._layouts.get(key)
        if paged is None:
            if len(self._layouts) >= 1024:
                self._layouts.clear()
            paged = describe_paged(kv_layer, self.block_size)
            self._layouts[key] = paged
        return paged

    def _done(self, future: Future[bool]) -> None:
        self._slots.release()

    # ------------------------------------------------------------- publish
    def publish_host_batch(self, pending: list[tuple[Any, int, int]], host: torch.Tensor) -> bool:
        """Publish each chunk of a chunk-major host batch as a view (no host copy)."""
        views = host.unbind(0)
        layer_id = pending[0][1] if pending else 0
        if all(layer == layer_id for _, layer, _ in pending):
            results = self.store.put_layers_host([sid for sid, _, _ in pending], layer_id,
                                                 views[: len(pending)])
        else:
            results = [self.store.put_layer_host(sid, layer, views[i])
                       for i, (sid, layer, _) in enumerate(pending)]
        committed = False
        for result in results:
            if result is not None:
                committed |= result
        return committed

    def publish_arena_batch(self, pending: list[tuple[Any, int, int]], slots: list,
                            chunk_shape: tuple[int, ...], dtype: torch.dtype) -> bool:
        """Publish each copied chunk as a view of its arena slot; dropped chunks (no
        slot) were already released by the reservation."""
        arena = self.store.arena
        layer_id = pending[0][1] if pending else 0
        kept = [(sid, slot) for (sid, _, _), slot in zip(pending, slots) if slot is not None]
        sids = [sid for sid, _ in kept]
        views = arena.layer_views([slot for _, slot in kept], layer_id, tuple(chunk_shape), dtype)
        results = self.store.put_layers_host(sids, layer_id, views) if sids else []
        return any(result for result in results if result is not None)

    def _publish_after_event(
        self,
        event: torch.cuda.Event,
        pending: list[tuple[Any, int, int]],
        host: torch.Tensor | None,
        request_id: str | None = None,
        store_enqueued_ns: int | None = None,
        arena_slots: list | None = None,
        chunk_shape: tuple[int, ...] = (),
        dtype: torch.dtype | None = None,
    ) -> bool:
        try:
            event.synchronize()
            if arena_slots is not None:
                committed = self.publish_arena_batch(pending, arena_slots, chunk_shape, dtype)
            else:
                committed = self.publish_host_batch(pending, host)
            if self.tracer.enabled:
                self.tracer.emit(
                    "save_store_finished",
                    request_id=request_id,
                    layer_id=pending[0][1] if pending else None,
                    chunks=len(pending),
                    tokens=sum(length for _, _, length in pending),
                    duration_us=(
                        (time.monotonic_ns() - store_enqueued_ns) / 1000
                        if store_enqueued_ns is not None
                        else None
                    ),
                    committed_segment=committed,
                )
            return committed
        except Exception:
            for segment_id, _, _ in pending:
                self.store.abort_put(segment_id)
            return False

    # ---------------------------------------------------------------- wait
    def wait_for_save(self) -> dict[str, int]:
        """Store stream drained and every publication joined; returns stores per request."""
        futures: tuple[Future[bool], ...] = ()
        counts: dict[str, int] = {}
        try:
            self.stream.synchronize()
            with self._lock:
                futures = tuple(self._futures)
                counts = dict(self._pending_counts)
                self._pending_counts.clear()
            for future in futures:
                future.result()
        finally:
            with self._lock:
                self._futures.difference_update(futures)
            # gathers and D2H copies are ordered on the Store stream, so the
            # staging may only be released after the synchronization above
            self._staging.clear()
            self._retired.clear()
            self._slot_cache.clear()
        return counts

    def drain(self) -> None:
        try:
            while True:
                with self._lock:
                    futures = tuple(self._futures)
                if not futures:
                    return
                for future in futures:
                    future.result()
                with self._lock:
                    self._futures.difference_update(futures)
        finally:
            self._staging.clear()
            self._retired.clear()
            self._slot_cache.clear()

    def close(self) -> None:
        try:
            self.drain()
        finally:
            self._layouts.clear()
            self._pool.shutdown(wait=True, cancel_futures=False)
