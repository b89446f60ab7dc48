"""``CacheBlendConnectorV1`` -- the vLLM V1 KV-connector plugin on B200.

Drop-in for cacheblend_vllm/connector.py:75-932: the same class name, the same
``kv_connector_extra_config`` fields, the same worker and scheduler methods
with the same request lifecycle.  The worker side runs the B200 hot path:
``start_load_kv`` drives ``Qwen3BlendExecutor`` over a ``PagedBlendLoader``
(layerwise H2D + fused load kernel + commit scatter, deviation / Sparse-Q
scoring, cluster top-k), and ``save_kv_layer`` feeds the ``StorePipeline``
(chunk-major gather + one D2H per batch + publication into the LRU).

The scheduler side keeps the reference's planning rules (APC-first plans,
gating, Sparse-Q span extension, slot mapping across chunked prefill,
cancellation).  Lookups go through a ``lookup`` object with
``lookup_and_prefetch(request_id, scope, tokens, apc)`` and ``cancel`` --
``LocalStoreLookup`` serves single-process deployments from the worker
stores; the reference's cross-process ZeroMQ lookup server is control plane
and can be plugged in through the same two methods.
"""

from __future__ import annotations

import math
import re
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any

import torch
from vllm.distributed.kv_transfer.kv_connector.v1.base import (
    KVConnectorBase_V1,
    KVConnectorMetadata,
    KVConnectorRole,
    SupportsHMA,
)

from . import registry
from .arena import PinnedArena
from .config import CacheBlendConfig
from .executor import Qwen3BlendExecutor
from .kv_layout import describe_paged
from .loader import PagedBlendLoader
from .storage import LocalPinnedCPUStore
from .store_path import StorePipeline
from .trace import PipelineTracer
from .types import BlendPlan, BlendSegment, SegmentId


def _slot_mapping(block_ids: list[int], block_size: int, token_count: int) -> torch.Tensor:
    """Token slots of a request's blocks, truncated to ``token_count``."""
    blocks = torch.tensor(block_ids, dtype=torch.long)
    return (blocks[:, None] * block_size + torch.arange(block_size)[None, :]).flatten()[:token_count]


def _layer_sort_key(name: str) -> tuple[int, str]:
    numbers = re.findall(r"(?:layers?\.)?(\d+)", name)
    return (int(numbers[-1]) if numbers else 1 << 30, name)


@dataclass(slots=True)
class RequestMetadata:
    request_id: str
    token_ids: list[int]
    slot_mapping: torch.Tensor
    plan: BlendPlan | None
    save: bool
    save_end: int


@dataclass(slots=True)
class _SchedulerRequestState:
    request: Any
    block_ids: list[int]
    cacheable: bool


@dataclass(slots=True)
class CacheBlendConnectorMetadata(KVConnectorMetadata):
    requests: list[RequestMetadata] = field(default_factory=list)


class LocalStoreLookup:
    """Lookup against the worker stores registered in this process.

    The protocol of the reference's tensor-parallel lookup
    (cacheblend_vllm/ipc.py:185-280): rank 0 matches the suffix after the APC
    prefix, the other ranks keep the subset they hold committed, every rank
    pins the intersection, and a rank that could not pin all of it cancels
    the whole request.
    """

    def __init__(self, engine_id: str):
        self.engine_id = engine_id

    def lookup_and_prefetch(self, request_id: str, model_scope: str, tokens: list[int],
                            start_offset: int) -> tuple[BlendSegment, ...]:
        stores = registry.stores(self.engine_id)
        if not stores:
            return ()
        candidates = tuple(
            BlendSegment(seg.segment_id, seg.target_start + start_offset)
            for seg in stores[0].match(model_scope, tokens[start_offset:], 0)
        )
        if not candidates:
            return ()
        common = set(candidates)
        for store in stores[1:]:
            common.intersection_update(store.validate(candidates))
        final = tuple(sorted(common, key=lambda seg: seg.target_start))
        if not final:
            return ()
        pinned = set(final)
        for store in stores:
            pinned.intersection_update(store.pin(request_id, final))
        if pinned != set(final):
            self.cancel(request_id)
            return ()
        return final

    def cancel(self, request_id: str) -> None:
        for store in registry.stores(self.engine_id):
            store.release(request_id)

    def close(self) -> None:
        return


SUPPORTED_VLLM = ((0, 22),)


def verify_runtime(strict: bool) -> None:
    """Fail fast on a vLLM whose V1 connector API this module was not written against."""
    if not strict:
        return
    try:
        from importlib.metadata import PackageNotFoundError, version

        found = version("vllm")
    except PackageNotFoundError:
        return
    match = re.match(r"^(\d+)\.(\d+)", found)
    if match is not None and (int(match.group(1)), int(match.group(2))) not in SUPPORTED_VLLM:
        raise RuntimeError(
            f"the B200 CacheBlend connector supports vLLM {SUPPORTED_VLLM}, found {found}. "
            "Set strict_version_check=false only for compatibility development."
        )


class CacheBlendConnectorV1(KVConnectorBase_V1, SupportsHMA):
    """APC-first, non-contiguous CacheBlend on B200 kernels."""

    @classmethod
    def requires_piecewise_for_cudagraph(cls, extra_config: dict[str, Any]) -> bool:
        # only decode-cache storage needs Python between graph pieces
        return bool(extra_config.get("save_decode_cache", False))

    def __init__(self, vllm_config, role: KVConnectorRole, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        transfer = vllm_config.kv_transfer_config
        assert transfer is not None
        self.config = CacheBlendConfig.from_extra_config(transfer.kv_connector_extra_config)
        verify_runtime(self.config.strict_version_check)
        self._recompute_on_failure = getattr(transfer, "kv_load_failure_policy", None) == "recompute"
        self.engine_id = str(transfer.engine_id)
        # a producer-only instance saves chunks and never blends: it needs no model
        self.kv_role = str(getattr(transfer, "kv_role", None) or "kv_both")
        self.block_size = int(vllm_config.cache_config.block_size)
        self.tp_size = int(vllm_config.parallel_config.tensor_parallel_size)
        if int(vllm_config.parallel_config.pipeline_parallel_size) != 1:
            raise ValueError("CacheBlendConnectorV1 currently requires pipeline_parallel_size=1")
        self.model_scope = self.config.model_scope or self._make_model_scope(vllm_config)
        self._init_state(role)
        if role is KVConnectorRole.SCHEDULER:
            self._lookup = LocalStoreLookup(self.engine_id)
            # one ordered background client keeps lookups off the scheduler thread
            self._lookup_pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="cacheblend-lookup")

    def _init_state(self, role) -> None:
        self._lookup = None
        self._lookup_pool: ThreadPoolExecutor | None = None
        self._lookup_futures: dict[str, Future] = {}
        self._lookup_state_lock = threading.Lock()
        self._cancelled_lookup_ids: set[str] = set()
        self._plans: dict[str, BlendPlan] = {}
        self._load_requests: dict[str, Any] = {}
        self._request_objects: dict[str, Any] = {}
        self._scheduler_requests: dict[str, _SchedulerRequestState] = {}
        self._store: LocalPinnedCPUStore | None = None
        self._kv_caches: list = []
        self._layer_ids: dict[str, int] = {}
        self._executor: Qwen3BlendExecutor | None = None
        self._load_errors: set[int] = set()
        self._save_segments: dict[str, list[tuple[int, SegmentId]]] = {}
        self._load_stream: torch.cuda.Stream | None = None
        self._pipeline: StorePipeline | None = None
        self._rank = 0
        component = "scheduler" if role is KVConnectorRole.SCHEDULER else "worker"
        self._trace = PipelineTracer(component)
        self._trace.emit("connector_initialized", engine_id=self.engine_id, model_scope=self.model_scope,
                         role=str(role), tp_size=self.tp_size)

    @staticmethod
    def _make_model_scope(vllm_config) -> str:
        model_config = vllm_config.model_config
        model = str(getattr(model_config, "model", "unknown-model"))
        revision = str(getattr(model_config, "revision", ""))
        dtype = str(getattr(model_config, "dtype", "unknown"))
        return f"{model}@{revision}|{dtype}|tp={int(vllm_config.parallel_config.tensor_parallel_size)}"

    # ================================================================ worker
    def register_kv_caches(self, kv_caches: dict[str, Any]) -> None:
        if self.role is not KVConnectorRole.WORKER:
            return
        ordered = sorted(kv_caches.items(), key=lambda item: _layer_sort_key(item[0]))
        self._layer_ids = {name: index for index, (name, _) in enumerate(ordered)}
        self._kv_caches = [value for _, value in ordered]
        if not self._kv_caches:
            raise RuntimeError("CacheBlendConnectorV1 received no KV caches")
        try:
            from vllm.distributed.parallel_state import get_tensor_model_parallel_rank

            self._rank = int(get_tensor_model_parallel_rank())
        except (AssertionError, ImportError):
            self._rank = 0
        self._store = LocalPinnedCPUStore(self.config.chunk_size, self.config.max_local_cpu_bytes)
        arena = self._make_arena()
        if arena is not None:
            self._store.attach_arena(arena)
        registry.register_store(self.engine_id, self._rank, self._store)
        first = self._kv_caches[0]
        device = (first if isinstance(first, torch.Tensor) else first[0]).device
        if device.type != "cuda":
            raise RuntimeError("the B200 CacheBlend connector needs CUDA KV caches")
        self._load_stream = torch.cuda.Stream(device=device)
        self._pipeline = StorePipeline(
            self._store, self.block_size, self.config.chunk_size, self.config.store_workers,
            self.config.max_inflight_store_batches, tracer=self._trace, device=device,
        )
        if self.kv_role != "kv_producer":
            self._executor = Qwen3BlendExecutor(registry.get_model(self.engine_id), self.config, self.block_size)
        self._trace.emit("worker_registered", rank=self._rank, layers=len(self._kv_caches),
                         cpu_cache_bytes=self.config.max_local_cpu_bytes)

    def _make_arena(self):
        """A pinned arena sized by ``local_cpu_gb`` when every layer has the same chunk
        geometry (one entry = every layer of one chunk); None otherwise (hybrid caches
        keep per-batch pinned buffers)."""
        geometry = set()
        for cache in self._kv_caches:
            paged = describe_paged(cache, self.block_size)
            geometry.add((tuple(paged.row.dims), paged.dtype))
        if len(geometry) != 1:
            return None
        dims, dtype = geometry.pop()
        layer_bytes = 2 * self.config.chunk_size * math.prod(dims) * torch.empty((), dtype=dtype).element_size()
        if layer_bytes * len(self._kv_caches) > self.config.max_local_cpu_bytes:
            return None
        return PinnedArena(layer_bytes, len(self._kv_caches), self.config.max_local_cpu_bytes)

    def start_load_kv(self, forward_context, **kwargs: Any) -> None:
        metadata = self._get_connector_metadata()
        if not isinstance(metadata, CacheBlendConnectorMetadata):
            raise TypeError("unexpected CacheBlend connector metadata")
        if self._store is None or self._executor is None:
            if any(request.plan is not None for request in metadata.requests):
                raise RuntimeError("CacheBlend worker was not initialized")
            return
        for request in metadata.requests:
            if request.plan is None:
                continue
            started = time.monotonic_ns() if self._trace.enabled else 0
            if self._trace.enabled:
                plan = request.plan
                self._trace.emit("blend_started", request_id=request.request_id,
                                 apc_prefix_tokens=plan.apc_prefix_tokens,
                                 allocation_tokens=plan.allocation_tokens, hit_tokens=plan.hit_tokens,
                                 gap_tokens=plan.gap_tokens, segments=len(plan.segments))
            loader = PagedBlendLoader(
                self._kv_caches, self._store, request.request_id, request.plan, request.slot_mapping,
                self.block_size, self.config, tracer=self._trace, load_stream=self._load_stream,
            )
            saved_moe = getattr(forward_context, "moe_layer_index", None)
            has_layer_idx = hasattr(forward_context, "layer_idx")
            saved_layer_idx = getattr(forward_context, "layer_idx", None)
            error: str | None = None
            try:
                self._executor.run(request.request_id, request.token_ids, request.plan, loader)
            except Exception as exc:
                error = type(exc).__name__
                self._record_load_error(request)
                if not self._recompute_on_failure:
                    raise
            finally:
                if hasattr(forward_context, "moe_layer_index"):
                    forward_context.moe_layer_index = saved_moe
                if has_layer_idx:
                    forward_context.layer_idx = saved_layer_idx
                self._store.release(request.request_id)
                if self._trace.enabled:
                    self._trace.emit("blend_finished", request_id=request.request_id,
                                     duration_us=(time.monotonic_ns() - started) / 1000, error=error)

    def wait_for_layer_load(self, layer_name: str) -> None:
        return

    def _resolve_layer(self, layer_name: str) -> int | None:
        layer_id = self._layer_ids.get(layer_name)
        if layer_id is not None:
            return layer_id
        key = _layer_sort_key(layer_name)[0]
        return next((i for name, i in self._layer_ids.items() if _layer_sort_key(name)[0] == key), None)

    def save_kv_layer(self, layer_name: str, kv_layer: Any, attn_metadata: Any, **kwargs: Any) -> None:
        if self._store is None:
            return
        metadata = self._get_connector_metadata()
        if not isinstance(metadata, CacheBlendConnectorMetadata):
            return
        layer_id = self._resolve_layer(layer_name)
        if layer_id is None:
            return
        chunk = self.config.chunk_size
        for request in metadata.requests:
            if not request.save:
                continue
            usable = min(request.save_end, len(request.token_ids), request.slot_mapping.numel())
            usable = usable // chunk * chunk
            segments = self._request_save_segments(request, usable)
            reserved = self._store.reserve_layers([sid for _, sid in segments], layer_id)
            pending: list[tuple[Any, int, int]] = []
            starts: list[int] = []
            for (start, segment_id), ok in zip(segments, reserved):
                if not ok:
                    continue
                pending.append((segment_id, layer_id, chunk))
                starts.append(start)
            if not pending:
                continue
            if starts[-1] - starts[0] == (len(starts) - 1) * chunk:
                # consecutive chunks (the usual case): one view, no concatenation
                slots = request.slot_mapping[starts[0] : starts[-1] + chunk]
            else:
                slots = torch.cat([request.slot_mapping[s : s + chunk] for s in starts])
            started = time.monotonic_ns() if self._trace.enabled else 0
            try:
                assert self._pipeline is not None
                self._pipeline.enqueue(pending, kv_layer, slots, request.request_id,
                                       store_enqueued_ns=started if self._trace.enabled else None)
                if self._trace.enabled:
                    self._trace.emit("save_store_enqueued", request_id=request.request_id,
                                     layer_id=layer_id, chunks=len(pending),
                                     tokens=len(pending) * chunk,
                                     duration_us=(time.monotonic_ns() - started) / 1000)
            except Exception:
                for segment_id, _, _ in pending:
                    self._store.abort_put(segment_id)
                raise

    def _request_save_segments(self, request: RequestMetadata, usable: int) -> list[tuple[int, SegmentId]]:
        """Content-addressed chunk ids, built once per request."""
        assert self._store is not None
        chunk = self.config.chunk_size
        segments = self._save_segments.setdefault(request.request_id, [])
        start = len(segments) * chunk
        missing = (usable - start) // chunk
        if missing > 0:
            ids = self._store.begin_put_chunks(self.model_scope, start, request.token_ids, missing,
                                               len(self._kv_caches))
            segments.extend((start + i * chunk, segment_id) for i, segment_id in enumerate(ids))
        return segments[: usable // chunk]

    def wait_for_save(self) -> None:
        started = time.monotonic_ns() if self._trace.enabled else 0
        counts = self._pipeline.wait_for_save() if self._pipeline is not None else {}
        if self._trace.enabled:
            duration = (time.monotonic_ns() - started) / 1000
            for request_id, stores in counts.items():
                self._trace.emit("save_store_wait_finished", request_id=request_id, stores=stores,
                                 duration_us=duration)

    def get_finished(self, finished_req_ids: set[str]) -> tuple[set[str] | None, set[str] | None]:
        if self._store is not None:
            for request_id in finished_req_ids:
                self._store.release(request_id)
                for _, segment_id in self._save_segments.pop(request_id, ()):
                    self._store.abort_put(segment_id)
        return None, None

    def get_block_ids_with_load_errors(self) -> set[int]:
        result, self._load_errors = self._load_errors, set()
        return result

    def _record_load_error(self, request: RequestMetadata) -> None:
        if request.plan is None:
            return
        slots = request.slot_mapping[request.plan.apc_prefix_tokens : request.plan.allocation_end]
        self._load_errors.update(int(v) for v in torch.unique(slots // self.block_size))

    # ============================================================= scheduler
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> tuple[int | None, bool]:
        if self.role is not KVConnectorRole.SCHEDULER:
            return 0, False
        request_id = request.request_id
        with self._lookup_state_lock:
            self._cancelled_lookup_ids.discard(request_id)
        self._request_objects[request_id] = request
        if not self._is_cacheable(request) or getattr(self, "kv_role", "kv_both") == "kv_producer":
            return 0, False
        plan = self._plans.get(request_id)
        if plan is not None:
            return max(0, plan.allocation_end - num_computed_tokens), False
        future = self._lookup_futures.get(request_id)
        if future is None:
            tokens = list(request.prompt_token_ids or [])
            if len(tokens) - num_computed_tokens <= self.config.chunk_size:
                self._plans[request_id] = BlendPlan(num_computed_tokens, num_computed_tokens, 0, ())
                return 0, False
            assert self._lookup_pool is not None
            self._lookup_futures[request_id] = self._lookup_pool.submit(
                self._lookup_plan, request_id, tokens, num_computed_tokens
            )
            return None, True
        if not future.done():
            return None, True
        del self._lookup_futures[request_id]
        try:
            plan = future.result()
        except Exception as exc:
            self._trace.emit("lookup_failed", request_id=request_id, error=type(exc).__name__)
            plan = BlendPlan(num_computed_tokens, num_computed_tokens, 0, ())
        self._plans[request_id] = plan
        return max(0, plan.allocation_end - num_computed_tokens), False

    def _lookup_plan(self, request_id: str, tokens: list[int], apc_prefix_tokens: int) -> BlendPlan:
        assert self._lookup is not None
        trace = self._trace.enabled
        started = time.monotonic_ns() if trace else 0
        if trace:
            self._trace.emit("lookup_started", request_id=request_id, prompt_tokens=len(tokens),
                             apc_prefix_tokens=apc_prefix_tokens)
        empty = BlendPlan(apc_prefix_tokens, apc_prefix_tokens, 0, ())

        def finished(outcome: str, plan: BlendPlan | None) -> None:
            if not trace:
                return
            fields = {"segments": 0, "hit_tokens": 0} if plan is None else {
                "segments": len(plan.segments), "allocation_tokens": plan.allocation_tokens,
                "hit_tokens": plan.hit_tokens, "gap_tokens": plan.gap_tokens}
            self._trace.emit("lookup_finished", request_id=request_id,
                             duration_us=(time.monotonic_ns() - started) / 1000, outcome=outcome,
                             apc_prefix_tokens=apc_prefix_tokens, **fields)

        # one prompt token stays with vLLM's regular step: search tokens[:-1]
        segments = self._lookup.lookup_and_prefetch(request_id, self.model_scope, tokens[:-1],
                                                    apc_prefix_tokens)
        with self._lookup_state_lock:
            cancelled = request_id in self._cancelled_lookup_ids
        if cancelled:
            # cleanup already queued a cancel behind this lookup
            finished("cancelled", None)
            return empty
        plan = BlendPlan.from_segments(apc_prefix_tokens, segments)
        if plan.segments and self.config.selection_strategy in {"sparse_q", "compare"}:
            # Sparse-Q must see the trailing non-reused question as queries
            plan = BlendPlan(plan.apc_prefix_tokens, len(tokens) - 1, plan.hit_tokens, plan.segments)
        if not plan.passes_gate(self.config.min_retrieve_tokens, self.config.min_hit_ratio,
                                self.config.min_saved_tokens, self.config.max_apc_prefix_to_hit_ratio):
            self._lookup.cancel(request_id)
            finished("rejected", plan)
            return empty
        finished("accepted", plan)
        return plan

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        if num_external_tokens <= 0:
            return
        if self._plans.get(request.request_id) is None:
            raise RuntimeError(f"missing CacheBlend plan for {request.request_id}")
        self._load_requests[request.request_id] = request

    @staticmethod
    def _is_cacheable(request) -> bool:
        # token ids alone do not identify these inputs
        return (
            getattr(request, "lora_request", None) is None
            and not getattr(request, "mm_features", None)
            and getattr(request, "prompt_embeds", None) is None
        )

    @staticmethod
    def _all_token_ids(request) -> list[int]:
        for name in ("all_token_ids", "_all_token_ids", "prompt_token_ids"):
            values = getattr(request, name, None)
            if values is not None:
                return list(values)
        return []

    def _save_end(self, request, computed_after_step: int, token_count: int) -> int:
        if self.config.save_decode_cache:
            return min(computed_after_step, token_count)
        return min(computed_after_step, len(getattr(request, "prompt_token_ids", None) or ()), token_count)

    def build_connector_meta(self, scheduler_output) -> CacheBlendConnectorMetadata:
        metadata = CacheBlendConnectorMetadata()
        emitted: set[str] = set()
        for request_id in scheduler_output.finished_req_ids:
            self._scheduler_requests.pop(request_id, None)
        for request_id in scheduler_output.preempted_req_ids or ():
            state = self._scheduler_requests.get(request_id)
            if state is not None:
                state.block_ids.clear()
        for new in scheduler_output.scheduled_new_reqs:
            request = self._request_objects.get(new.req_id)
            token_ids = self._all_token_ids(request) if request is not None else list(new.prompt_token_ids or [])
            num_tokens = min(len(token_ids), len(new.block_ids[0]) * self.block_size)
            plan = self._plans.get(new.req_id)
            if new.req_id in self._load_requests:
                emitted.add(new.req_id)
            else:
                plan = None
            cacheable = request is not None and self._is_cacheable(request)
            if request is not None:
                self._scheduler_requests[new.req_id] = _SchedulerRequestState(
                    request, list(new.block_ids[0]), cacheable
                )
            computed_after = new.num_computed_tokens + scheduler_output.num_scheduled_tokens[new.req_id]
            metadata.requests.append(RequestMetadata(
                request_id=new.req_id,
                token_ids=token_ids,
                slot_mapping=_slot_mapping(new.block_ids[0], self.block_size, num_tokens),
                plan=plan,
                save=cacheable,
                save_end=self._save_end(request, computed_after, num_tokens) if request is not None else 0,
            ))
        cached = scheduler_output.scheduled_cached_reqs
        for index, request_id in enumerate(cached.req_ids):
            state = self._scheduler_requests.get(request_id)
            if state is None:
                continue
            new_blocks = cached.new_block_ids[index]
            if new_blocks is not None:
                if request_id in cached.resumed_req_ids:
                    state.block_ids = list(new_blocks[0])
                else:
                    state.block_ids.extend(new_blocks[0])
            if not state.block_ids:
                continue
            token_ids = self._all_token_ids(state.request)
            num_tokens = min(len(token_ids), len(state.block_ids) * self.block_size)
            computed_after = cached.num_computed_tokens[index] + scheduler_output.num_scheduled_tokens[request_id]
            metadata.requests.append(RequestMetadata(
                request_id=request_id,
                token_ids=token_ids,
                slot_mapping=_slot_mapping(state.block_ids, self.block_size, num_tokens),
                plan=self._plans.get(request_id) if request_id in self._load_requests else None,
                save=state.cacheable,
                save_end=self._save_end(state.request, computed_after, num_tokens),
            ))
            if request_id in self._load_requests:
                emitted.add(request_id)
        for request_id in emitted:
            self._load_requests.pop(request_id, None)
        return metadata

    def request_finished(self, request, block_ids: list[int]) -> tuple[bool, dict[str, Any] | None]:
        self._cleanup_scheduler_request(request.request_id)
        return False, None

    def request_finished_all_groups(self, request, block_ids) -> tuple[bool, dict[str, Any] | None]:
        self._cleanup_scheduler_request(request.request_id)
        return False, None

    def _cleanup_scheduler_request(self, request_id: str) -> None:
        future = self._lookup_futures.pop(request_id, None)
        if future is not None and not future.cancel():
            with self._lookup_state_lock:
                self._cancelled_lookup_ids.add(request_id)
        self._plans.pop(request_id, None)
        self._load_requests.pop(request_id, None)
        self._request_objects.pop(request_id, None)
        self._scheduler_requests.pop(request_id, None)
        if self._lookup is not None and self._lookup_pool is not None:
            self._lookup_pool.submit(self._cancel_lookup, request_id)

    def _cancel_lookup(self, request_id: str) -> None:
        if self._lookup is not None:
            self._lookup.cancel(request_id)
        with self._lookup_state_lock:
            self._cancelled_lookup_ids.discard(request_id)

    def close(self) -> None:
        try:
            if self._pipeline is not None:
                self._pipeline.close()
                self._pipeline = None
        finally:
            if self._lookup_pool is not None:
                self._lookup_pool.shutdown(wait=True, cancel_futures=False)
                self._lookup_pool = None
            if self._lookup is not None:
                self._lookup.close()
                self._lookup = None
            if self._store is not None:
                registry.unregister_store(self.engine_id, self._rank)
                self._store.clear()
            self._trace.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001 - destructors must never raise
            return
