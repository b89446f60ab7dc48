"""Layerwise blend load into double-buffered staging (K2 + host-link pipeline).

Drop-in for ``PagedBlendLoader`` (cacheblend_vllm/ascend.py:170-407): same
constructor, ``prefetch(layer_id, rotary_emb)``, ``get(layer_id)`` and
``commit(layer_id, contiguous)``, same staging contents (APC prefix gathered
from pages, gaps zeroed, hit chunks relocated from their source to their
target positions), same double buffering with reuse events, same trace
events.  Per layer the B200 path is:

* host -> device: the layer's hit chunks reach the GPU either by copy-engine
  DMA (one ``cudaMemcpyAsync`` per run of host-adjacent chunks into a packed
  device hit buffer) or, in zero-copy mode, not as a separate step at all --
  the load kernel reads the pinned host chunks directly over the host link;
* one ``cb_blend_load_layer`` launch writes the whole staging buffer (prefix
  gather + gap zeros + relocated K + copied V);
* ``commit`` is one ``cb_paged_scatter`` launch of the suffix.

The mode comes from ``CACHEBLEND_B200_LOAD`` (``copy`` | ``zerocopy``);
zero-copy uses copy mode for a layer whose chunks are not all pinned.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch

from . import _native
from .config import CacheBlendConfig
from .kv_layout import PagedKV, RowShape, dense_row, describe_paged, device_slots, scatter_from
from .rope import cos_sin_table, relocate_key, rope_geometry
from .storage import LocalPinnedCPUStore
from .trace import PipelineTracer
from .types import BlendPlan

LOAD_MODE_ENV = "CACHEBLEND_B200_LOAD"
# CTAs of a zero-copy load: enough 16-byte loads in flight to cover host-link
# latency x bandwidth, few enough to leave the serving stream the other SMs.
ZERO_COPY_CTAS = 64


def load_mode() -> str:
    mode = os.getenv(LOAD_MODE_ENV, "copy").strip().lower()
    if mode not in ("copy", "zerocopy"):
        raise ValueError(f"{LOAD_MODE_ENV} must be 'copy' or 'zerocopy', got {mode!r}")
    return mode


def rope_head_stride(row: RowShape, rope_head_bytes: int) -> int:
    """Byte stride between consecutive RoPE heads of a KV row."""
    if row.num_heads == 1:
        if row.row_bytes % rope_head_bytes:
            raise ValueError("KV row is not a whole number of RoPE heads")
        return rope_head_bytes
    if row.head_bytes != rope_head_bytes:
        raise ValueError("KV cache heads do not match the RoPE head size")
    return row.head_stride


_COPY_STREAMS: dict[int, torch.cuda.Stream] = {}


def _copy_stream(device: torch.device) -> torch.cuda.Stream:
    """One host->device copy stream per device, shared by all loaders."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    stream = _COPY_STREAMS.get(index)
    if stream is None:
        stream = torch.cuda.Stream(device=index)
        _COPY_STREAMS[index] = stream
    return stream


def byte_span(tensor: torch.Tensor, nbytes: int) -> torch.Tensor:
    """uint8 view of ``nbytes`` bytes of ``tensor``'s storage from its first element."""
    offset = tensor.storage_offset() * tensor.element_size()
    return torch.empty(0, dtype=torch.uint8).set_(
        tensor.untyped_storage(), offset, (nbytes,), (1,)
    )


class PagedBlendLoader:
    """Double-buffered layerwise CPU -> GPU blend load and paged-cache commit."""

    def __init__(
        self,
        kv_caches: list[torch.Tensor | tuple[torch.Tensor, torch.Tensor]],
        store: LocalPinnedCPUStore,
        request_id: str,
        plan: BlendPlan,
        slot_mapping: torch.Tensor,
        block_size: int,
        config: CacheBlendConfig,
        tracer: PipelineTracer | None = None,
        load_stream: torch.cuda.Stream | None = None,
    ):
        self.kv_caches = kv_caches
        self.store = store
        self.request_id = request_id
        self.plan = plan
        self.slot_mapping = slot_mapping[: plan.allocation_end]
        self.block_size = block_size
        self.config = config
        self.tracer = tracer
        self.mode = load_mode()
        self._buffers: dict[int, torch.Tensor] = {}
        self._events: dict[int, torch.cuda.Event] = {}
        self._reuse_events: dict[int, torch.cuda.Event] = {}
        self._staging: list[torch.Tensor] = []
        # copy mode: two device hit buffers (layer parity) so the H2D of layer
        # l+1 on the copy stream overlaps the load kernel of layer l
        self._hit_buffers: list[torch.Tensor | None] = [None, None]
        self._copy_tables: list[torch.Tensor | None] = [None, None]
        self._hit_free: dict[int, torch.cuda.Event] = {}
        self._slots: torch.Tensor | None = None
        self._device_error: torch.Tensor | None = None
        self._token_segment: torch.Tensor | None = None
        self._host_refs: list[torch.Tensor] = []  # sources of in-flight host reads
        old, new = plan.hit_positions()
        self._old_positions_cpu = torch.from_numpy(old)
        self._new_positions_cpu = torch.from_numpy(new)
        if config.fused_segment_copy:
            # all hits relocate together; skipped only if no position moves
            moved = bool(np.any(old != new))
            self._rotate = np.full(len(plan.segments), int(moved), dtype=np.int32)
        else:
            # per-segment relocation, skipped where source == target
            self._rotate = np.array(
                [int(seg.source_start != seg.target_start) for seg in plan.segments],
                dtype=np.int32,
            )
        self._load_stream = load_stream if config.event_pipeline else None
        if self.tracer is not None and self.tracer.enabled:
            self.tracer.emit(
                "loader_initialized",
                request_id=request_id,
                apc_prefix_tokens=plan.apc_prefix_tokens,
                allocation_tokens=plan.allocation_tokens,
                hit_tokens=plan.hit_tokens,
                gap_tokens=plan.gap_tokens,
                segments=len(plan.segments),
            )

    # ------------------------------------------------------------------ setup
    def _setup(self, paged: PagedKV) -> None:
        if self._slots is None:
            self._device_error = torch.zeros(1, dtype=torch.int32, device=paged.device)
            self._slots = device_slots(self.slot_mapping, paged, self.block_size)
            segment_map = torch.from_numpy(self.plan.token_segment_map())
            self._token_segment = segment_map.to(paged.device, non_blocking=True)
        if not self._staging:
            shape = (2, self.plan.allocation_end, *paged.row.dims)
            self._staging = [
                torch.empty(shape, dtype=paged.dtype, device=paged.device) for _ in range(2)
            ]

    # ------------------------------------------------------------- host side
    def _base_table(self) -> np.ndarray:
        segments = self.plan.segments
        table = np.zeros(len(segments), dtype=_native.SEGMENT_DTYPE)
        table["source_start"] = [seg.source_start for seg in segments]
        table["target_start"] = [seg.target_start for seg in segments]
        table["length"] = [seg.length for seg in segments]
        table["rotate"] = self._rotate
        return table

    def _check_host(self, host: torch.Tensor, paged: PagedKV, length: int) -> None:
        expected = (2, length, *paged.row.dims)
        if tuple(host.shape) != expected or host.dtype != paged.dtype:
            raise ValueError(
                f"stored chunk has shape {tuple(host.shape)} {host.dtype}, expected {expected}"
            )

    def _segment_table(
        self, paged: PagedKV, layer_id: int, rope_head_bytes: int, kernel_rotates: bool
    ) -> tuple[torch.Tensor | None, bool]:
        """This layer's device cb_segment_t table and whether it reads host memory."""
        segments = self.plan.segments
        if not segments:
            return None, False
        get_layers = getattr(self.store, "get_layers", None)
        if get_layers is not None:  # one lock acquisition for the layer's segments
            hosts = get_layers(self.request_id, segments, layer_id)
        else:
            hosts = [self.store.get_layer(self.request_id, seg, layer_id) for seg in segments]
        for host, seg in zip(hosts, segments, strict=True):
            self._check_host(host, paged, seg.length)
        zero_copy = self.mode == "zerocopy" and all(host.is_pinned() for host in hosts)
        parity = layer_id % 2
        if not zero_copy:
            self._copy_hits(hosts, paged, parity)
            cached = self._copy_tables[parity]
            if cached is not None and kernel_rotates:
                return cached, False
        table = self._base_table()
        if not kernel_rotates:
            table["rotate"] = 0
        esize = paged.row.element_size
        row_bytes = paged.row.row_bytes
        if zero_copy:
            for index, host in enumerate(hosts):
                table["k_src"][index] = host[0].data_ptr()
                table["v_src"][index] = host[1].data_ptr()
                table["src_token_stride"][index] = host.stride(1) * esize
                table["src_head_stride"][index] = rope_head_stride(dense_row(host), rope_head_bytes)
            self._host_refs.extend(hosts)
        else:
            hit_buffer = self._hit_buffers[parity]
            assert hit_buffer is not None
            offsets = np.cumsum([0] + [2 * seg.length * row_bytes for seg in segments[:-1]])
            lengths = np.array([seg.length for seg in segments], dtype=np.int64)
            base = hit_buffer.data_ptr()
            table["k_src"] = (base + offsets).astype(np.uint64)
            table["v_src"] = (base + offsets + lengths * row_bytes).astype(np.uint64)
            table["src_token_stride"] = row_bytes
            table["src_head_stride"] = rope_head_bytes
        device_table = torch.from_numpy(table.view(np.uint8)).pin_memory().to(
            paged.device, non_blocking=True
        )
        if not zero_copy and kernel_rotates:
            self._copy_tables[parity] = device_table  # identical for every layer of this parity
        return device_table, zero_copy

    def _copy_hits(self, hosts: list[torch.Tensor], paged: PagedKV, parity: int) -> None:
        """Copy-engine H2D of every hit chunk into the packed device hit buffer.

        Per segment the buffer holds its K plane then its V plane.  Pieces that
        are adjacent in one pinned host allocation (chunk-major Store batches)
        move as a single copy.  With an event pipeline the copies run on a
        dedicated copy stream: they wait until the load kernel two layers back
        has released this parity's buffer, and the load stream waits for them.
        """
        row_bytes = paged.row.row_bytes
        total = sum(2 * host.shape[1] * row_bytes for host in hosts)
        hit_buffer = self._hit_buffers[parity]
        if hit_buffer is None or hit_buffer.numel() < total:
            hit_buffer = torch.empty(total, dtype=torch.uint8, device=paged.device)
            self._hit_buffers[parity] = hit_buffer
            self._copy_tables[parity] = None
        runs: list[list] = []  # [first piece, dst offset, bytes, next src ptr, storage ptr]
        pinned: dict[int, bool] = {}  # per host storage: pinned (queried once per storage)
        offset = 0
        for host in hosts:
            pieces = [host] if host.is_contiguous() else [host[0], host[1]]
            for piece in pieces:
                if not piece.is_contiguous():
                    piece = piece.contiguous()
                nbytes = piece.numel() * piece.element_size()
                ptr = piece.data_ptr()
                storage = piece.untyped_storage().data_ptr()
                last = runs[-1] if runs else None
                if last is not None and last[3] == ptr and last[4] == storage:
                    is_pinned = pinned.get(storage)
                    if is_pinned is None:
                        is_pinned = pinned[storage] = piece.is_pinned()
                    if is_pinned:
                        last[2] += nbytes
                        last[3] += nbytes
                        offset += nbytes
                        continue
                runs.append([piece, offset, nbytes, ptr + nbytes, storage])
                offset += nbytes
        load_stream = torch.cuda.current_stream()
        copy_stream = _copy_stream(paged.device) if self._load_stream is not None else load_stream
        if copy_stream is not load_stream:
            free = self._hit_free.pop(parity, None)
            if free is not None:
                copy_stream.wait_event(free)
        with torch.cuda.stream(copy_stream):
            for piece, dst_offset, nbytes, _, _ in runs:
                src = byte_span(piece, nbytes)
                hit_buffer[dst_offset : dst_offset + nbytes].copy_(src, non_blocking=True)
                self._host_refs.append(src)
        if copy_stream is not load_stream:
            copied = torch.cuda.Event()
            copied.record(copy_stream)
            load_stream.wait_event(copied)

    # ----------------------------------------------------------- public API
    def prefetch(self, layer_id: int, rotary_emb) -> None:
        if layer_id in self._buffers or layer_id >= len(self.kv_caches):
            return
        trace = self.tracer is not None and self.tracer.enabled
        started = time.monotonic_ns() if trace else 0
        paged = describe_paged(self.kv_caches[layer_id], self.block_size)
        _native.require_cuda(paged.key)
        stream = self._load_stream if self._load_stream is not None else torch.cuda.current_stream()
        with torch.cuda.stream(stream):
            self._setup(paged)
            index = layer_id % 2
            reuse = self._reuse_events.pop(index, None)
            if reuse is not None:
                stream.wait_event(reuse)
            buffer = self._staging[index]
            self._launch_load(layer_id, paged, buffer, rotary_emb, stream)
            if self._load_stream is not None:
                event = torch.cuda.Event()
                event.record(stream)
                self._events[layer_id] = event
                self._hit_free[index] = event  # this parity's hit buffer is consumed
        self._buffers[layer_id] = buffer
        if trace:
            assert self.tracer is not None
            self.tracer.emit(
                "layer_prefetch_enqueued",
                request_id=self.request_id,
                layer_id=layer_id,
                duration_us=(time.monotonic_ns() - started) / 1000,
            )

    def _launch_load(
        self,
        layer_id: int,
        paged: PagedKV,
        buffer: torch.Tensor,
        rotary_emb,
        stream: torch.cuda.Stream,
    ) -> None:
        plan = self.plan
        head_size, rotary_dim, neox = rope_geometry(rotary_emb)
        esize = paged.row.element_size
        rope_head_bytes = head_size * esize
        kernel_rotates = hasattr(rotary_emb, "cos_sin_cache")
        table = cos_sin_table(rotary_emb, paged.dtype, paged.device) if kernel_rotates else None
        device_table, zero_copy = self._segment_table(
            paged, layer_id, rope_head_bytes, kernel_rotates
        )
        num_heads = paged.row.row_bytes // rope_head_bytes
        paged_hs = rope_head_stride(paged.row, rope_head_bytes)
        _native.call(
            "cb_blend_load_layer",
            buffer.data_ptr(),
            buffer.stride(0) * esize,
            buffer.stride(1) * esize,
            rope_head_bytes,
            plan.allocation_end,
            plan.apc_prefix_tokens,
            paged.key.data_ptr(),
            paged.value.data_ptr(),
            paged.block_stride,
            paged.slot_stride,
            paged_hs,
            paged.num_blocks,
            self.block_size,
            self._slots.data_ptr(),
            num_heads,
            head_size,
            _native.dtype_code(paged.dtype),
            self._token_segment.data_ptr(),
            0 if device_table is None else device_table.data_ptr(),
            len(plan.segments),
            0 if table is None else table.data_ptr(),
            0 if table is None else table.shape[0],
            rotary_dim,
            int(neox),
            ZERO_COPY_CTAS if zero_copy else 0,
            self._device_error.data_ptr(),
            _native.stream_handle(stream),
        )
        if not kernel_rotates and self._rotate.any():
            self._relocate_with_module(buffer, rotary_emb, paged.device)

    def _relocate_with_module(self, buffer: torch.Tensor, rotary_emb, device) -> None:
        """Relocation through a rotary module that exposes no cos_sin_cache."""
        if self.config.fused_segment_copy:
            new = self._new_positions_cpu.to(device)
            old = self._old_positions_cpu.to(device)
            buffer[0, new] = relocate_key(rotary_emb, old, new, buffer[0, new])
            return
        for seg, rotate in zip(self.plan.segments, self._rotate, strict=True):
            if not rotate:
                continue
            rows = slice(seg.target_start, seg.target_end)
            old = torch.arange(seg.source_start, seg.source_start + seg.length, device=device)
            new = torch.arange(seg.target_start, seg.target_end, device=device)
            buffer[0, rows] = relocate_key(rotary_emb, old, new, buffer[0, rows])

    def device_error(self) -> int:
        """Pipeline timeout code reported by the load kernels (0 = none); synchronizes."""
        return 0 if self._device_error is None else int(self._device_error.item())

    def get(self, layer_id: int) -> torch.Tensor:
        event = self._events.pop(layer_id, None)
        if event is not None:
            torch.cuda.current_stream().wait_event(event)
        if self.tracer is not None and self.tracer.enabled:
            self.tracer.emit(
                "layer_prefetch_wait_enqueued",
                request_id=self.request_id,
                layer_id=layer_id,
                had_event=event is not None,
            )
        return self._buffers.pop(layer_id)

    def commit(self, layer_id: int, contiguous: torch.Tensor) -> None:
        start = self.plan.apc_prefix_tokens
        if start >= self.plan.allocation_end:
            return
        paged = describe_paged(self.kv_caches[layer_id], self.block_size)
        self._setup(paged)
        assert self._slots is not None
        scatter_from(contiguous[:, start:], paged, self._slots[start:])
        if self._load_stream is not None:
            event = torch.cuda.Event()
            event.record(torch.cuda.current_stream())
            self._reuse_events[layer_id % 2] = event
        if self.tracer is not None and self.tracer.enabled:
            self.tracer.emit(
                "layer_committed",
                request_id=self.request_id,
                layer_id=layer_id,
                suffix_tokens=self.plan.allocation_end - start,
            )
