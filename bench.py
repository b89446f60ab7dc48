"""Benchmark of the CacheBlend B200 hot path (load + score + scatter).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2]

One step = one blend request carried through every layer of the model:
per layer the fused blend load (APC prefix gather + gap zeroing + RoPE
relocation + placement of the reused chunks into staging), at the check layer
the K-deviation score + recompute top-k, and the commit scatter of the
recomputed span into vLLM pages.  Default workload: Qwen3-8B shapes (36
layers, 8 KV heads, head_dim 128, bf16), a 32,768-token prompt in 128 chunks
of 256 with 89 reused chunks at random non-contiguous positions, block_size
16, kv_deviation at layer 1 with ratio 0.15.  Synthetic data
(seeded N(0,1) bf16); the model math between load and commit is not part of
the path and is not run.

* ``value``  -- blend-span tokens/s with the reused chunks already in HBM.
* ``e2e``    -- the same request through the public ``PagedBlendLoader`` API
  with the chunks in a pinned ``LocalPinnedCPUStore``: per layer H2D of the
  reused chunks inside the timed region, and the selected indices read back.
* ``roofline`` -- dominant kernel's algorithmic bytes / CUDA-event time vs the
  measured HBM copy bandwidth.
* ``cpu_baseline`` -- the CPU restatement (oracle/, OpenMP) on a bounded
  sample of the same workload, extrapolated to the full request.

With ``--gpus N`` (torchrun, one rank per GPU) the KV heads are split over N
tensor-parallel ranks (8/N heads each), the deviation scores are all-reduced
over NCCL and every rank selects the same tokens; work per request is fixed
("strong" scaling).  ``--impl reference`` times the CPU restatement on the
host cores with the same metric (rank 0 only).
"""

from __future__ import annotations

import argparse
import ctypes
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "pic-kvcache_b200"))
sys.path.insert(0, str(REPO))

METRIC = "blend-span tokens/s (load+score+scatter)"
UNIT = "tokens/s"
L2_BYTES = 126 * (1 << 20)


@dataclass(frozen=True)
class Shape:
    name: str
    layers: int
    kv_heads: int
    q_heads: int
    head_dim: int
    tokens: int
    chunk: int
    hit_chunks: int
    block_size: int
    pool_blocks: int
    max_position: int
    rope_theta: float
    check_layer: int
    ratio: float


SPARSE_Q_CONFIG = {"name": "qwen3-30b-a3b-98k-sparse_q", "layers": 48, "q_heads": 32, "kv_heads": 4,
                   "head_dim": 128, "tokens": 98304, "query_chunks": 16, "check_layer": 6}

ATTENTION_CONFIG = {"name": "qwen3-8b-32k-blend_attention", "q_heads": 32, "kv_heads": 8, "head_dim": 128,
                    "tokens": 32768, "ratio": 0.15}

ATTENTION_KEYS = 0  # --attention-tokens: a smaller context for profiling captures

STORE_CONFIG = {"name": "qwen3-8b-store-64x8k", "layers": 36, "kv_heads": 8, "head_dim": 128, "requests": 64,
                "tokens": 8192, "chunk": 256, "block_size": 16, "local_cpu_gb": 16.0, "inflight": 8,
                "workers": 1}

CONFIGS = {
    1: Shape("qwen3-0.6b-cpu-plumbing", 28, 8, 16, 128, 4096, 256, 12, 16, 2048, 40960, 1e6, 1, 0.15),
    2: Shape("qwen3-8b-32k-kv_deviation", 36, 8, 32, 128, 32768, 256, 89, 16, 2304, 40960, 1e6, 1, 0.15),
    # a 64K prompt needs a RoPE table past Qwen3-32B's native 40,960 positions: vLLM builds
    # 131,072 for the YaRN-extended (factor 4) context
    4: Shape("qwen3-32b-64k-kv_deviation", 64, 8, 64, 128, 65536, 256, 192, 16, 4352, 131072, 1e6, 1, 0.15),
}


def make_plan(shape: Shape, seed: int):
    """Seeded plan: reused chunks at random chunk slots, random source offsets."""
    from cacheblend_b200.types import BlendPlan, BlendSegment, SegmentId

    if shape.tokens > shape.max_position:
        # target rows past the RoPE table would be zero-filled (fail closed), not relocated
        raise ValueError(f"{shape.name}: {shape.tokens} tokens exceed the RoPE table ({shape.max_position})")
    rng = np.random.default_rng(seed)
    chunks = shape.tokens // shape.chunk
    hits = np.sort(rng.choice(chunks, size=shape.hit_chunks, replace=False))
    segments = []
    for i, c in enumerate(hits):
        source = int(rng.integers(0, shape.max_position - shape.chunk))
        sid = SegmentId("bench", 1_000_003 * i + 17, source, shape.chunk)
        segments.append(BlendSegment(sid, int(c) * shape.chunk))
    return BlendPlan.from_segments(0, segments)


def rope_table(shape: Shape, device) -> torch.Tensor:
    """vLLM-style fp32 cos_sin_cache [max_position, head_dim] (neox)."""
    inv = 1.0 / (shape.rope_theta ** (torch.arange(0, shape.head_dim, 2, dtype=torch.float64) / shape.head_dim))
    freqs = torch.arange(shape.max_position, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).float().to(device)


class Rope:
    def __init__(self, shape: Shape, device):
        self.head_size = shape.head_dim
        self.rotary_dim = shape.head_dim
        self.is_neox_style = True
        self.cos_sin_cache = rope_table(shape, device)


class Workload:
    """Device pages, device-resident hit chunks and a pinned host store for one rank."""

    def __init__(self, shape: Shape, tp: int, rank: int, device, seed: int = 2, host_store: bool = True):
        from cacheblend_b200.config import CacheBlendConfig
        from cacheblend_b200.storage import LocalPinnedCPUStore

        assert shape.kv_heads % tp == 0, "KV heads must divide over the TP ranks"
        self.shape = shape
        self.heads = shape.kv_heads // tp
        self.device = device
        self.plan = make_plan(shape, seed)
        self.gen = torch.Generator(device=device).manual_seed(seed * 7919 + rank)
        rng = np.random.default_rng(seed)
        hd = shape.head_dim
        row = self.heads * hd
        self.row_bytes = row * 2
        self.pages = [
            torch.randn(2, shape.pool_blocks, shape.block_size, self.heads, hd, generator=self.gen,
                        device=device, dtype=torch.bfloat16)
            for _ in range(shape.layers)
        ]
        blocks = rng.permutation(shape.pool_blocks)[: shape.tokens // shape.block_size]
        slots = (blocks[:, None] * shape.block_size + np.arange(shape.block_size)[None, :]).reshape(-1)
        self.slot_mapping = torch.from_numpy(slots.astype(np.int64))
        self.rope = Rope(shape, device)
        self.config = CacheBlendConfig.from_extra_config(
            {"check_layers": [shape.check_layer], "recompute_ratios": [shape.ratio],
             "chunk_size": shape.chunk, "strict_version_check": False}
        )
        plan = self.plan
        nseg = len(plan.segments)
        # device-resident hit chunks: [layers, segments, 2, chunk, heads, hd]
        self.hits = torch.randn(shape.layers, nseg, 2, shape.chunk, self.heads, hd, generator=self.gen,
                                device=device, dtype=torch.bfloat16)
        self.act = plan.allocation_end - plan.apc_prefix_tokens
        cached = torch.empty(self.act, row, device=device, dtype=torch.bfloat16)
        self.fresh_noise = (torch.randn(self.act, row, generator=self.gen, device=device) * 0.05)
        self.gap_mask = plan.gap_mask()[plan.apc_prefix_tokens:]
        del cached
        self.store = None
        if host_store:
            self.store = LocalPinnedCPUStore(shape.chunk, max_bytes=(nseg + 1) * shape.layers * 2
                                             * shape.chunk * self.row_bytes, pin_memory=True)
            self._publish(nseg)

    def _publish(self, nseg: int) -> None:
        """Fill the pinned store: one chunk-major pinned batch per layer."""
        shape = self.shape
        tokens = {}
        for i, seg in enumerate(self.plan.segments):
            tokens[i] = list(range(i * shape.chunk, (i + 1) * shape.chunk))
        ids = []
        for i, seg in enumerate(self.plan.segments):
            sid = self.store.begin_put("bench", seg.source_start, tokens[i], shape.layers)
            ids.append(sid)
        self.host_batches = []
        for layer in range(shape.layers):
            batch = torch.empty(self.hits[layer].shape, dtype=torch.bfloat16, pin_memory=True)
            batch.copy_(self.hits[layer])
            self.host_batches.append(batch)
            for i, sid in enumerate(ids):
                self.store.put_layer_host(sid, layer, batch[i])
        from cacheblend_b200.types import BlendPlan, BlendSegment

        segments = [BlendSegment(sid, seg.target_start) for sid, seg in zip(ids, self.plan.segments)]
        self.store_plan = BlendPlan.from_segments(self.plan.apc_prefix_tokens, segments)
        pinned = self.store.pin("bench-request", segments)
        assert len(pinned) == len(segments)

    def device_tables(self):
        """Per-layer cb_segment_t tables pointing at the device-resident hits."""
        from cacheblend_b200 import _native

        plan = self.plan
        segs = plan.segments
        moved = any(s.source_start != s.target_start for s in segs)
        tables = []
        for layer in range(self.shape.layers):
            table = np.zeros(len(segs), dtype=_native.SEGMENT_DTYPE)
            base = self.hits[layer].data_ptr()
            seg_bytes = 2 * self.shape.chunk * self.row_bytes
            for i, seg in enumerate(segs):
                table[i] = (base + i * seg_bytes, base + i * seg_bytes + self.shape.chunk * self.row_bytes,
                            self.row_bytes, self.shape.head_dim * 2, seg.source_start, seg.target_start,
                            seg.length, int(moved))
            tables.append(torch.from_numpy(table.view(np.uint8)).to(self.device))
        return tables


def open_peer_exchange(group, max_tokens: int, device):
    """The TP group's peer-memory score exchange, or None (every rank alike) when a rank
    cannot create or map its buffer: the NCCL all-reduce then sums the scores."""
    from cacheblend_b200.peer_exchange import PeerExchangeUnavailable, PeerScoreExchange

    try:
        return PeerScoreExchange(group, max_tokens, device)
    except PeerExchangeUnavailable as error:
        print(f"peer score exchange unavailable, using the NCCL all-reduce: {error}", file=sys.stderr)
        return None


class DevicePath:
    """The hot path straight through the C ABI with device-resident inputs."""

    def __init__(self, wl: Workload, tp_group=None):
        from cacheblend_b200 import _native
        from cacheblend_b200.kv_layout import describe_paged
        from cacheblend_b200.rope import cos_sin_table

        self.wl = wl
        self.native = _native
        self.tp_group = tp_group
        shape = wl.shape
        plan = wl.plan
        dev = wl.device
        self.tables = wl.device_tables()
        self.paged = [describe_paged(p, shape.block_size) for p in wl.pages]
        self.slots = wl.slot_mapping[: plan.allocation_end].to(dev)
        self.token_segment = torch.from_numpy(plan.token_segment_map()).to(dev)
        self.cos_sin = cos_sin_table(wl.rope, torch.bfloat16, dev)
        self.staging = [torch.empty(2, plan.allocation_end, wl.heads, shape.head_dim, dtype=torch.bfloat16,
                                    device=dev) for _ in range(2)]
        self.scores = torch.empty(wl.act, dtype=torch.float32, device=dev)
        self.device_error = torch.zeros(1, dtype=torch.int32, device=dev)
        base = np.asarray(wl.gap_mask, dtype=np.uint8)
        self.base_mask = torch.from_numpy(base).to(dev)
        from cacheblend_b200.selection import recompute_budget

        gaps = int(base.sum())
        self.k = recompute_budget(wl.act, gaps, gaps, shape.ratio)
        self.selected = torch.empty(gaps + self.k, dtype=torch.long, device=dev)
        # fresh K for the check layer = cached hits + noise, prepared once
        self.fresh = None
        # the check layer's deviation and select: two launches (with TP the score all-reduce
        # sits between them); CACHEBLEND_B200_FUSED_SELECT=1 times the single fused launch
        # (cb_kv_deviation_select) on one rank instead
        self.fused = tp_group is None and os.environ.get("CACHEBLEND_B200_FUSED_SELECT") == "1"
        # with TP the score reduction runs inside the select kernel over NVLink peer memory
        # (cb_select_topk_peer); CACHEBLEND_B200_PEER_SELECT=0 puts the NCCL all-reduce back
        self.peer = None
        if tp_group is not None and os.environ.get("CACHEBLEND_B200_PEER_SELECT", "1") != "0":
            self.peer = open_peer_exchange(tp_group, wl.act, dev)
        self.fused_workspace = None
        if self.fused:
            size = ctypes.c_int64(0)
            self.native.call("cb_kv_deviation_select_workspace_size", ctypes.addressof(size))
            self.fused_workspace = torch.zeros(size.value, dtype=torch.uint8, device=dev)
        score_kinds = ["deviation_select"] if self.fused else ["deviation", "select"]
        self.events: dict[str, list] = {name: [] for name in ["load", "scatter", *score_kinds]}
        self.timing = False
        self.graphs: list = []
        self.side = torch.cuda.Stream(dev)  # the loader's Load stream in the pipelined step

    def _ev(self, name: str, stream):
        if not self.timing:
            return None
        start = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        return start

    def _ev_end(self, name: str, start, stream):
        if start is None:
            return
        end = torch.cuda.Event(enable_timing=True)
        end.record(stream)
        self.events[name].append((start, end))

    def load_layer(self, layer: int, stream) -> torch.Tensor:
        wl, shape, plan = self.wl, self.wl.shape, self.wl.plan
        buf = self.staging[layer % 2]
        pg = self.paged[layer]
        h = stream.cuda_stream
        ev = self._ev("load", stream)
        self.native.call(
            "cb_blend_load_layer", buf.data_ptr(), buf.stride(0) * 2, buf.stride(1) * 2, shape.head_dim * 2,
            plan.allocation_end, plan.apc_prefix_tokens, pg.key.data_ptr(), pg.value.data_ptr(),
            pg.block_stride, pg.slot_stride, shape.head_dim * 2, pg.num_blocks, shape.block_size,
            self.slots.data_ptr(), wl.heads, shape.head_dim, 0, self.token_segment.data_ptr(),
            self.tables[layer].data_ptr(), len(plan.segments), self.cos_sin.data_ptr(),
            self.cos_sin.shape[0], shape.head_dim, 1, 0, self.device_error.data_ptr(), h,
        )
        self._ev_end("load", ev, stream)
        return buf

    def score(self, buf: torch.Tensor, stream) -> torch.Tensor:
        if self.fused:
            return self.deviation_select(buf, stream)
        self.deviation(buf, stream)
        if self.tp_group is not None and self.peer is None:
            torch.distributed.all_reduce(self.scores, group=self.tp_group)
        return self.select(stream)

    def deviation(self, buf: torch.Tensor, stream) -> None:
        wl, shape, plan = self.wl, self.wl.shape, self.wl.plan
        if self.fresh is None:
            k_plane = buf[0].reshape(plan.allocation_end, -1)
            self.fresh = (k_plane[plan.apc_prefix_tokens:].float() + wl.fresh_noise).to(torch.bfloat16)
        width = wl.heads * shape.head_dim
        ev = self._ev("deviation", stream)
        self.native.call(
            "cb_kv_deviation", self.fresh.data_ptr(), width * 2, buf.data_ptr(), width * 2,
            plan.allocation_end, 0,
            plan.apc_prefix_tokens, wl.act, width, 0, self.scores.data_ptr(), stream.cuda_stream,
        )
        self._ev_end("deviation", ev, stream)

    def _fresh_for(self, buf: torch.Tensor) -> torch.Tensor:
        wl, plan = self.wl, self.wl.plan
        if self.fresh is None:
            k_plane = buf[0].reshape(plan.allocation_end, -1)
            self.fresh = (k_plane[plan.apc_prefix_tokens:].float() + wl.fresh_noise).to(torch.bfloat16)
        return self.fresh

    def deviation_select(self, buf: torch.Tensor, stream, rotation: tuple | None = None) -> torch.Tensor:
        """The check layer's deviation and select in one launch (one rank)."""
        wl, shape, plan = self.wl, self.wl.shape, self.wl.plan
        fresh = self._fresh_for(buf)
        cached = buf
        if rotation is not None:
            fresh, cached = rotation
        width = wl.heads * shape.head_dim
        ev = self._ev("deviation_select", stream)
        self.native.call(
            "cb_kv_deviation_select", fresh.data_ptr(), width * 2, cached.data_ptr(), width * 2,
            plan.allocation_end, 0, plan.apc_prefix_tokens, wl.act, width, 0, self.base_mask.data_ptr(),
            self.k, self.scores.data_ptr(), self.selected.data_ptr(), self.selected.numel(),
            self.fused_workspace.data_ptr(), self.fused_workspace.numel(), stream.cuda_stream,
        )
        self._ev_end("deviation_select", ev, stream)
        return self.selected

    def deviation_rotating(self, index: int, rotation: list, stream) -> None:
        """The check layer's deviation launch on the ``index``-th copy of its inputs."""
        wl, shape, plan = self.wl, self.wl.shape, self.wl.plan
        fresh, k_plane = rotation[index]
        width = wl.heads * shape.head_dim
        self.native.call(
            "cb_kv_deviation", fresh.data_ptr(), width * 2, k_plane.data_ptr(), width * 2,
            plan.allocation_end, 0, plan.apc_prefix_tokens, wl.act, width, 0, self.scores.data_ptr(),
            stream.cuda_stream,
        )

    def select(self, stream) -> torch.Tensor:
        wl = self.wl
        ev = self._ev("select", stream)
        if self.peer is not None:
            self.peer.select(self.scores, self.base_mask, self.k, self.selected.numel(), stream,
                             out=self.selected)
        else:
            self.native.call(
                "cb_select_topk", self.scores.data_ptr(), self.base_mask.data_ptr(), wl.act, self.k,
                self.selected.data_ptr(), self.selected.numel(), stream.cuda_stream,
            )
        self._ev_end("select", ev, stream)
        return self.selected

    def commit(self, layer: int, buf: torch.Tensor, stream) -> None:
        wl, shape, plan = self.wl, self.wl.shape, self.wl.plan
        pg = self.paged[layer]
        start = plan.apc_prefix_tokens
        n = plan.allocation_end - start
        ev = self._ev("scatter", stream)
        self.native.call(
            "cb_paged_scatter", buf[:, start:].data_ptr(), buf.stride(0) * 2, buf.stride(1) * 2,
            shape.head_dim * 2, 0, 0, pg.key.data_ptr(), pg.value.data_ptr(), pg.block_stride,
            pg.slot_stride, shape.head_dim * 2, pg.num_blocks, shape.block_size, wl.heads,
            shape.head_dim * 2, self.slots[start:].data_ptr(), n, stream.cuda_stream,
        )
        self._ev_end("scatter", ev, stream)

    def step(self, stream) -> None:
        if self.graphs:
            self.graphs[0].replay()
            if len(self.graphs) == 2:
                torch.distributed.all_reduce(self.scores, group=self.tp_group)
                self.graphs[1].replay()
            return
        for layer in range(self.wl.shape.layers):
            buf = self.load_layer(layer, stream)
            if layer == self.wl.shape.check_layer:
                self.score(buf, stream)
            self.commit(layer, buf, stream)

    def _pipelined(self, main, part: str) -> None:
        """The step's launches as the loader pipelines them: loads on a side stream (the
        loader's Load stream), scoring and commits on the main stream, load(l) before
        commit(l), commit(l-2) before load(l) (the two staging buffers alternate), so the
        load of layer l+1 runs beside the commit of layer l.  ``part``: "all" layers, or
        "until" / "after" the check layer's scores (TP: the all-reduce sits in between)."""
        # Overlap only pays for rows under 2 KiB: there the kernels are short enough that
        # each one's ramp and tail dominate; with 2 KiB rows both kernels fill HBM and the
        # SMs on their own (measured on B200: 3.67 vs 3.16 ms per request at 8 heads).
        side = self.side if self.wl.row_bytes < 2048 else main
        layers, check = self.wl.shape.layers, self.wl.shape.check_layer
        first = check + 1 if part == "after" else 0
        last = check if part == "until" else layers - 1
        if side is not main:
            side.wait_stream(main)  # fork
        committed: dict[int, torch.cuda.Event] = {}

        def done(stream) -> torch.cuda.Event:
            ev = torch.cuda.Event()
            ev.record(stream)
            return ev

        if part == "after":
            self.select(main)
            self.commit(check, self.staging[check % 2], main)
            if side is not main:
                committed[check] = done(main)
        for layer in range(first, last + 1):
            if side is not main and layer - 2 in committed:
                side.wait_event(committed[layer - 2])
            with torch.cuda.stream(side):
                self.load_layer(layer, side)
            if side is not main:
                main.wait_event(done(side))
            if layer == check:
                if self.fused:
                    self.deviation_select(self.staging[layer % 2], main)
                else:
                    self.deviation(self.staging[layer % 2], main)
                    if part == "until" and self.peer is None:
                        break
                    self.select(main)
            self.commit(layer, self.staging[layer % 2], main)
            if side is not main:
                committed[layer] = done(main)
        if side is not main:
            main.wait_stream(side)  # join

    def capture(self, stream) -> None:
        """CUDA graphs of the pipelined step (no per-launch host work while timing): one
        graph on a single rank or with the peer-memory select; with the NCCL all-reduce,
        two graphs around it."""
        assert self.fresh is not None and not self.timing
        torch.cuda.synchronize(self.wl.device)
        graphs = []
        for part in (["all"] if self.tp_group is None or self.peer is not None else ["until", "after"]):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                self._pipelined(stream, part)
            graphs.append(graph)
        self.graphs = graphs

    def release(self) -> None:
        self.graphs = []

    def close(self) -> None:
        """Free the peer exchange (every rank together)."""
        self.graphs = []
        if self.peer is not None:
            self.peer.check()
            self.peer.close()
            self.peer = None

    def kernel_graph_us(self, stream, reps: int = 20, sync=None) -> dict[str, float]:
        """Average launch duration of each kernel, back to back as in the step: one step's
        36 loads (resp. 36 commit scatters, or ten deviation / select launches) captured
        in a graph, replayed ``reps`` times between two CUDA events on the launching stream."""
        layers = self.wl.shape.layers
        check = self.wl.shape.check_layer
        k_plane = self.staging[check % 2][0]
        rotation = [(self.fresh.clone(), k_plane.clone()) for _ in range(4)]
        kinds = {
            "load": (layers, lambda: [self.load_layer(layer, stream) for layer in range(layers)]),
            "scatter": (layers, lambda: [self.commit(layer, self.staging[layer % 2], stream)
                                         for layer in range(layers)]),
        }
        # single launches per step: ten back to back over four rotating input sets (512 MiB
        # at 8 heads), so each launch reads its fresh and cached K from HBM, not from L2
        if self.fused:
            kinds["deviation_select"] = (10, lambda: [self.deviation_select(
                None, stream, rotation[i % len(rotation)]) for i in range(10)])
        else:
            kinds["deviation"] = (10, lambda: [self.deviation_rotating(i % len(rotation), rotation, stream)
                                               for i in range(10)])
            kinds["select"] = (10, lambda: [self.select(stream) for _ in range(10)])
        out = {}
        for name, (count, launch) in kinds.items():
            torch.cuda.synchronize(self.wl.device)
            if sync is not None:
                sync()  # TP: the ranks start each kind together (the peer select waits on the others)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                launch()
            with torch.cuda.stream(stream):
                graph.replay()
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record(stream)
                for _ in range(reps):
                    graph.replay()
                end.record(stream)
            end.synchronize()
            out[name] = start.elapsed_time(end) * 1e3 / (reps * count)
            del graph
        return out


def e2e_step(wl: Workload, load_stream, tp_group=None) -> tuple[torch.Tensor, int]:
    """One request through the public API: loader (H2D from the pinned store) + select."""
    from cacheblend_b200.loader import PagedBlendLoader
    from cacheblend_b200.selection import deviation_select, kv_deviation, select_tokens

    shape, plan = wl.shape, wl.store_plan
    loader = PagedBlendLoader(wl.pages, wl.store, "bench-request", plan, wl.slot_mapping,
                              shape.block_size, wl.config, load_stream=load_stream)
    loader.prefetch(0, wl.rope)
    selected = None
    for layer in range(shape.layers):
        buf = loader.get(layer)
        loader.prefetch(layer + 1, wl.rope)
        if layer == shape.check_layer:
            k_plane = buf[0].reshape(plan.allocation_end, -1)
            if not hasattr(wl, "e2e_fresh"):
                wl.e2e_fresh = (k_plane[plan.apc_prefix_tokens:].float() + wl.fresh_noise).to(torch.bfloat16)
            if tp_group is None and os.environ.get("CACHEBLEND_B200_FUSED_SELECT") == "1":
                selected, _ = deviation_select(wl.e2e_fresh, k_plane, wl.gap_mask, shape.ratio,
                                               absolute_offset=plan.apc_prefix_tokens)
            else:
                scores = kv_deviation(wl.e2e_fresh, k_plane, absolute_offset=plan.apc_prefix_tokens)
                selected = select_tokens(scores, wl.gap_mask, shape.ratio, tp_group=tp_group,
                                         peer_exchange=getattr(wl, "peer", None))
        loader.commit(layer, buf)
    host = selected.to("cpu")  # device -> host read of the step's result
    return host, host.numel() * host.element_size()


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------- helpers
def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data.get("bf16_tflops", 1590.0)),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_traffic() -> dict:
    """Per-launch DRAM bytes of the kernels from the committed ncu summary."""
    path = REPO / "profiles" / "traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


def algorithmic_bytes(wl: Workload) -> dict[str, float]:
    plan, rb = wl.plan, wl.row_bytes
    hits = plan.hit_tokens
    alloc = plan.allocation_end
    act = wl.act
    return {
        # read reused K+V rows (+ prefix rows), write the whole K+V staging
        "load": 2 * rb * (hits + plan.apc_prefix_tokens) + 2 * rb * alloc,
        # read staging suffix, write pages
        "scatter": 2 * (2 * rb * act),
        "deviation": 2 * rb * act + 4 * act,
        "select": 4 * act * 6 + act,
        # one pass over both K planes, the scores written and read back once by the last cluster
        "deviation_select": 2 * rb * act + 4 * act + 4 * act + act,
    }


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    group = None
    if world > 1:
        import datetime

        if args.impl == "ours":
            torch.cuda.set_device(local)
        torch.distributed.init_process_group(
            "nccl" if args.impl == "ours" else "gloo", timeout=datetime.timedelta(seconds=120),
            device_id=torch.device("cuda", local) if args.impl == "ours" else None,
        )
        group = torch.distributed.group.WORLD
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local, group


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()


# ---------------------------------------------------------------------------- CPU baseline
def host_link_peak(device, nbytes: int = 1 << 30, repeats: int = 3) -> dict:
    """Best-of-N single pinned<->device copy bandwidth (the host-link roofline)."""
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    out = {}
    for name, dst, src in (("h2d_gbs", dev, host), ("d2h_gbs", host, dev)):
        best = 0.0
        for _ in range(repeats):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            dst.copy_(src, non_blocking=True)
            end.record()
            end.synchronize()
            best = max(best, nbytes / (start.elapsed_time(end) / 1e3) / 1e9)
        out[name] = best
    del host, dev
    return out


def run_e2e(args, wl: Workload, device, world: int, group, span: int) -> dict:
    """Same request through the public loader API with the chunks in pinned host memory."""
    from cacheblend_b200.loader import load_mode

    shape = wl.shape
    load_stream = torch.cuda.Stream(device)
    for _ in range(2):
        e2e_step(wl, load_stream, tp_group=group)
    torch.cuda.synchronize(device)
    barrier(world)
    torch.cuda.synchronize(device)
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record()
    d2h = 0
    for _ in range(args.e2e_steps):
        _, d2h = e2e_step(wl, load_stream, tp_group=group)
    e_end.record()
    torch.cuda.synchronize(device)
    barrier(world)
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world, device) / args.e2e_steps
    h2d = len(wl.plan.segments) * shape.layers * 2 * shape.chunk * wl.row_bytes
    link = host_link_peak(device)
    achieved = h2d / (e2e_ms / 1e3) / 1e9
    return {"value": span / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": e2e_ms, "load_mode": load_mode(),
            "host_link": {"achieved_gbs": achieved, "peak_h2d_gbs": link["h2d_gbs"],
                          "peak_d2h_gbs": link["d2h_gbs"], "frac": achieved / link["h2d_gbs"],
                          "peak_source": "measured: best single 1 GiB pinned->device copy"}}


class CpuRequest:
    """The whole request on the host: the CPU restatement (oracle/, C + OpenMP) of
    every layer's blend load (APC prefix gather, gap zeroing, RoPE relocation,
    chunk placement: ascend.py:224-370) and commit scatter (kv_layout.py:125-161),
    plus the check layer's K-deviation and top-k select (ascend.py:534-543,
    757-796).  Inputs are generated once; ``run`` is one timed request."""

    def __init__(self, shape: Shape, threads: int, seed: int = 2):
        import oracle

        self.oracle = oracle
        self.shape = shape
        self.threads = threads
        self.plan = plan = make_plan(shape, seed)
        rng = np.random.default_rng(seed)
        hd, heads = shape.head_dim, shape.kv_heads
        self.row = heads * hd
        self.table = oracle.f32_to_bf16(rope_table(shape, "cpu").numpy())
        blocks = rng.permutation(shape.pool_blocks)[: shape.tokens // shape.block_size]
        slots = (blocks[:, None] * shape.block_size + np.arange(shape.block_size)[None, :]).reshape(-1)
        self.slots = slots[: plan.allocation_end].astype(np.int64)
        self.moved = np.full(len(plan.segments), 1, dtype=np.int32)
        # bf16 bit patterns with moderate exponents (no inf/NaN patterns)
        self.k = rng.integers(0, 1 << 16, size=(shape.pool_blocks, shape.block_size, heads, hd),
                              dtype=np.uint16) & 0xBFFF
        self.v = rng.integers(0, 1 << 16, size=self.k.shape, dtype=np.uint16) & 0xBFFF
        hosts = [rng.integers(0, 1 << 16, size=(2, shape.chunk, heads, hd), dtype=np.uint16) & 0xBFFF
                 for _ in plan.segments]
        self.segments = [(s.source_start, s.target_start, s.length, h) for s, h in zip(plan.segments, hosts)]
        self.act = plan.allocation_end - plan.apc_prefix_tokens
        self.gaps = plan.gap_mask()[plan.apc_prefix_tokens:]

    def run(self, layers: int | None = None) -> float:
        """Seconds for ``layers`` layers (default: all) and the check-layer scoring."""
        oracle, shape, plan = self.oracle, self.shape, self.plan
        start = plan.apc_prefix_tokens
        t0 = time.perf_counter()
        for layer in range(shape.layers if layers is None else layers):
            staging = oracle.blend_load(oracle.BF16, plan.allocation_end, start, self.k, self.v, self.slots,
                                        shape.block_size, self.segments, self.moved, self.table,
                                        shape.head_dim, shape.head_dim, True, self.threads)
            if layer == shape.check_layer or (layers is not None and layer == layers - 1):
                k_plane = staging[0].reshape(plan.allocation_end, self.row)
                scores = oracle.kv_deviation(k_plane[start:].copy(), k_plane, oracle.BF16, abs_offset=start,
                                             nthreads=self.threads)
                oracle.select(scores, self.gaps, shape.ratio)
            oracle.paged_scatter(staging[:, start:], self.k, self.v, self.slots[start:], shape.block_size)
        return time.perf_counter() - t0


def cpu_baseline(shape: Shape, threads: int, requests: int = 2) -> dict:
    """The CPU restatement timed on whole requests (best of ``requests``), no extrapolation."""
    request = CpuRequest(shape, threads)
    request.run(layers=1)  # warm the pages and the thread pool
    best = min(request.run() for _ in range(requests))
    return {"value": request.act / best, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"whole {shape.layers}-layer requests (best of {requests}): every layer's blend "
                      "load and commit scatter plus the check-layer deviation and select",
            "ms_per_request": best * 1e3}


def workload_config(shape: Shape, span: int, heads: int, world: int, shard: int) -> dict:
    """The ``config`` of the load+score+scatter lines (the GPU arm and the reference arm alike)."""
    row = heads * shape.head_dim * 2
    plan = make_plan(shape, 2)
    touched = 2 * row * (plan.hit_tokens + plan.apc_prefix_tokens) + 2 * row * plan.allocation_end + 4 * row * span
    return {"workload": shape.name, "tokens": shape.tokens, "span_tokens": span, "layers": shape.layers,
            "kv_heads_per_rank": heads, "hit_chunks": shape.hit_chunks, "block_size": shape.block_size,
            "check_layer": shape.check_layer, "ratio": shape.ratio,
            "parallelism": f"tp{world}" if shard == world else f"one rank of tp{shard}",
            "l2": f"inputs larger than L2 (each layer touches {touched / 2**20:.0f} MiB)"}


# ---------------------------------------------------------------------------- main
def run_reference(args, shape: Shape, world: int, rank: int) -> None:
    """--impl reference: the reference's CPU path (its restatement) on whole requests,
    all host threads; each timed step is one full request, nothing extrapolated."""
    if rank != 0:
        return
    import oracle

    threads = oracle.threads(0)
    request = CpuRequest(shape, threads)
    for _ in range(args.warmup):
        request.run(layers=1)
    times = [request.run() for _ in range(args.steps)]
    step_s = statistics.median(times)
    value = request.act / step_s
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16)",
        "config": workload_config(shape, request.act, shape.kv_heads // world, world, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"each step one whole {shape.layers}-layer request (median of "
                                   f"{args.steps}); warm-up steps run one layer"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def sparse_q_inputs(world: int, rank: int, device):
    """Config 3 inputs: 98,303 keys, 16 seeded gap chunks (4,095 queries) as the
    sparse queries, Q and K ~ N(0, 1) bf16, this rank's share of the heads."""
    cfg = SPARSE_Q_CONFIG
    hq, hkv = cfg["q_heads"] // world, cfg["kv_heads"] // world
    ctx = cfg["tokens"] - 1  # the last prompt token stays with vLLM (connector.py:664-673)
    rng = np.random.default_rng(3)
    gen = torch.Generator(device=device).manual_seed(30 + rank)
    chunks = rng.choice(ctx // 256, size=cfg["query_chunks"] - 1, replace=False)
    positions = np.sort(np.concatenate([c * 256 + np.arange(256) for c in chunks]
                                       + [np.arange((ctx // 256) * 256, ctx)]))
    key = torch.randn(ctx, hkv, 128, generator=gen, device=device).to(torch.bfloat16)
    query = torch.randn(ctx, hq, 128, generator=gen, device=device).to(torch.bfloat16)
    return ctx, positions, query, key


def sparse_q_cpu_sample(positions: np.ndarray, query, key, scale: float, flops: float,
                        budget_s: float = 12.0) -> dict:
    """The oracle's Sparse-Q (numpy, BLAS threads) on query chunks spread over the
    prompt until about ``budget_s``; scaled to the full step by algorithmic flops."""
    import oracle

    k = key.float().cpu().numpy()
    order = np.random.default_rng(7).permutation(positions.size // 8) * 8
    done_flops, done, t0 = 0.0, 0, time.perf_counter()
    for start in order:
        rows = positions[start:start + 8]
        q = query[torch.from_numpy(rows).to(query.device)].float().cpu().numpy()
        oracle.sparse_q_key_mass(q, k[: int(rows.max()) + 1], rows, scale)
        done_flops += float(sum(2 * 128 * query.shape[1] * (int(p) + 1) for p in rows))
        done += rows.size
        if time.perf_counter() - t0 > budget_s:
            break
    elapsed = time.perf_counter() - t0
    step_s = elapsed * flops / done_flops
    try:
        from threadpoolctl import threadpool_info

        cores = max([int(info.get("num_threads", 1)) for info in threadpool_info()] + [1])
    except ImportError:
        cores = 1
    return {"value": (key.shape[0]) / step_s, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{done} of {positions.size} queries (chunks of 8 spread over the prompt), numpy "
                      f"oracle with BLAS on {cores} threads, scaled to the step by algorithmic flops",
            "est_ms_per_step": step_s * 1e3}


def sparse_q_reference(args) -> None:
    """--impl reference for config 3: the reference's Sparse-Q (its numpy restatement)
    on the host, each step a bounded sample of the step's queries scaled by flops."""
    cfg = SPARSE_Q_CONFIG
    ctx, positions, query, key = sparse_q_inputs(1, 0, torch.device("cpu"))
    flops = float(sum(2 * 128 * cfg["q_heads"] * (int(p) + 1) for p in positions))
    samples = [sparse_q_cpu_sample(positions, query, key, 128 ** -0.5, flops, budget_s=2.0)
               for _ in range(args.warmup + args.steps)][args.warmup:]
    value = float(np.median([s["value"] for s in samples]))
    print(json.dumps({
        "impl": "reference", "metric": "sparse-q scored span tokens/s (boundary layer, TP-sharded)",
        "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ctx / value * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16)",
        "config": {"workload": cfg["name"], "keys": ctx, "queries": int(positions.size),
                   "q_heads_per_rank": cfg["q_heads"], "kv_heads_per_rank": cfg["kv_heads"]},
        "cpu_baseline": {**samples[-1], "value": value},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def sparse_q_bench(args, world: int, rank: int, local: int, steps: int, cpu: bool) -> dict | None:
    """Config 3: Sparse-Q scoring at the boundary layer (tensor-core bound) + select."""
    from cacheblend_b200.selection import select_tokens, sparse_q_key_mass, sparse_q_masks

    cfg = SPARSE_Q_CONFIG
    device = torch.device("cuda", local)
    ctx, positions, query, key = sparse_q_inputs(world, rank, device)
    hq, hkv = query.shape[1], key.shape[1]
    gaps = np.zeros(ctx, dtype=bool)
    gaps[positions] = True
    qmask, forced, _ = sparse_q_masks(gaps, 16, 1, 64)
    rows = np.flatnonzero(qmask)
    workspace = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    error = torch.zeros(1, dtype=torch.int32, device=device)
    scale = 128 ** -0.5
    flops = float(sum(2 * 128 * cfg["q_heads"] * (int(p) + 1) for p in positions)) / world

    # with TP the key masses are summed inside the select kernel over NVLink peer memory,
    # as the executor does (CACHEBLEND_B200_PEER_SELECT=0: NCCL all-reduce, then select)
    peer = None
    if world > 1 and os.environ.get("CACHEBLEND_B200_PEER_SELECT", "1") != "0":
        peer = open_peer_exchange(torch.distributed.group.WORLD, ctx, device)

    def step():
        mass = sparse_q_key_mass(query, key, rows, positions, scale, workspace=workspace, device_error=error)
        if world > 1 and peer is None:
            torch.distributed.all_reduce(mass)
        return select_tokens(mass, gaps, 0.15, forced, peer_exchange=peer)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(steps):
            step()
        end.record()
        torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, device) / steps
    if peer is not None:
        peer.check()
        peer.close()
    peaks = measured_peaks()
    peak = peaks["bf16_tflops"]
    achieved = flops / (ms / 1e3) / 1e12
    # co-limit: one exp2 per score element in each of the two passes on the MUFU
    # pipe (16 per SM per clock on B200)
    exps = 2.0 * flops / (2 * 128)
    mufu_peak = 16 * 148 * 1.965e9
    if rank != 0:
        return None
    cpu_line = None
    if cpu and world == 1:
        cpu_line = sparse_q_cpu_sample(positions, query, key, scale, flops)
    return {
        "metric": "sparse-q scored span tokens/s (boundary layer, TP-sharded)", "value": ctx / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16)",
        "config": {"workload": cfg["name"], "keys": ctx, "queries": int(positions.size),
                   "q_heads_per_rank": hq, "kv_heads_per_rank": hkv,
                   "l2": "K and the sparse queries re-streamed per tile pair; 201 MiB of K, larger than L2"},
        "gpu_launches": 4 * steps, "launch": "eager: query prep, row pass, key pass, select per step"
                                             + ("" if peer is None else " (the select sums the ranks' "
                                                                         "key masses over NVLink)"),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peaks["source"],
                     "flops_note": "one causal QK^T counted once (two passes run); timed over the step "
                                   "(prep, both passes, select)",
                     "co_limit": {"pipe": "mufu exp2", "achieved_per_s": exps / (ms / 1e3),
                                  "peak_per_s": mufu_peak, "frac": exps / (ms / 1e3) / mufu_peak,
                                  "peak_source": "16 exp2 per SM per clock x 148 SMs x 1965 MHz (nominal)"}},
        "device_error": int(error.item()), "clocks": clocks.summary(), "cpu_baseline": cpu_line,
    }


def attention_inputs(world: int, rank: int, device):
    """Config 6 inputs: the staging context of one layer (K / V rows = positions)
    and the queries of the rows kept after the check layer (15% of the span,
    the last prompt token among them), TP-sharded over heads."""
    cfg = ATTENTION_CONFIG
    ctx = (ATTENTION_KEYS or cfg["tokens"]) - 1
    rng = np.random.default_rng(6)
    count = int(round(cfg["ratio"] * ctx))
    positions = np.sort(np.concatenate([rng.choice(ctx - 1, size=count - 1, replace=False), [ctx - 1]]))
    hq, hkv = cfg["q_heads"] // world, cfg["kv_heads"] // world
    gen = torch.Generator(device=device).manual_seed(60 + rank)
    query = torch.randn(positions.size, hq, 128, generator=gen, device=device).to(torch.bfloat16)
    key = torch.randn(ctx, hkv, 128, generator=gen, device=device).to(torch.bfloat16)
    value = torch.randn(ctx, hkv, 128, generator=gen, device=device).to(torch.bfloat16)
    return positions, query, key, value


def attention_flops(positions: np.ndarray, q_heads: int) -> float:
    """Causal QK^T plus PV over keys <= position: 4 * head_dim per (query head, key)."""
    return 4.0 * 128 * q_heads * float((positions.astype(np.float64) + 1).sum())


def attention_bench(args, world: int, rank: int, local: int) -> None:
    """Config 6: the executor's attention of the kept rows over the staging
    context (one layer), on the tensor cores."""
    from cacheblend_b200.attention import attention_workspace_bytes, blend_attention

    cfg = ATTENTION_CONFIG
    device = torch.device("cuda", local)
    positions, query, key, value = attention_inputs(world, rank, device)
    pos = torch.from_numpy(positions).to(device)
    nq, hq = query.shape[0], query.shape[1]
    workspace = torch.empty(attention_workspace_bytes(nq, key.shape[0], hq, key.shape[1], 128, torch.bfloat16),
                            dtype=torch.uint8, device=device)
    error = torch.zeros(1, dtype=torch.int32, device=device)
    scale = 128 ** -0.5
    stream = torch.cuda.Stream(device)

    def step():
        return blend_attention(query, key, value, pos, scale, workspace=workspace, device_error=error,
                               stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.synchronize(device)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, device) / args.steps
    # the one-launch modes, same steps: the einsum roundings in flash order, and fp32
    # logits (the reference's fused NPU kernel semantics)
    other_ms = {}
    for mode in ("flash", "fused"):
        with torch.cuda.stream(stream):
            for _ in range(3):
                blend_attention(query, key, value, pos, scale, workspace=workspace, device_error=error,
                                stream=stream, exact_rounding=mode)
        torch.cuda.synchronize(device)
        barrier(world)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            f0.record(stream)
            for _ in range(args.steps):
                blend_attention(query, key, value, pos, scale, workspace=workspace, device_error=error,
                                stream=stream, exact_rounding=mode)
            f1.record(stream)
        torch.cuda.synchronize(device)
        barrier(world)
        other_ms[mode] = max_over_ranks(f0.elapsed_time(f1), world, device) / args.steps
    flops = attention_flops(positions, hq)
    # context: torch SDPA with the boolean causal-by-position mask (the generic path)
    allowed = pos[:, None] >= torch.arange(key.shape[0], device=device)[None, :]
    sdpa = lambda: torch.nn.functional.scaled_dot_product_attention(
        query.transpose(0, 1)[None], key.transpose(0, 1)[None], value.transpose(0, 1)[None],
        attn_mask=allowed[None, None], scale=scale, enable_gqa=hq != key.shape[1])
    sdpa()
    torch.cuda.synchronize(device)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(3):
        sdpa()
    s1.record()
    torch.cuda.synchronize(device)
    sdpa_ms = s0.elapsed_time(s1) / 3
    peaks = measured_peaks()
    peak = peaks["bf16_tflops"]
    achieved = flops / (ms / 1e3) / 1e12
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = attention_cpu_sample(positions, query, key, value, scale)
        print(json.dumps({
            "metric": "blend-attention query tokens/s (one layer, TP-sharded heads)",
            "value": positions.size / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16)",
            "config": {"workload": cfg["name"] + (f"-{ATTENTION_KEYS}tok" if ATTENTION_KEYS else ""),
                       "keys": int(key.shape[0]), "queries": int(positions.size),
                       "q_heads_per_rank": hq, "kv_heads_per_rank": int(key.shape[1]),
                       "l2": "inputs larger than L2 (K, V and Q: %d MiB)"
                             % ((key.numel() * 2 + query.numel()) * 2 >> 20)},
            "gpu_launches": 3 * args.steps,
            "launch": "eager (query prep, row log2-sum-exp, attention with normalized P per step)",
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": peaks["source"],
                         "traffic": load_traffic().get(f"{cfg['name']}:attention:tp{world}")
                         if not ATTENTION_KEYS else None,
                         "flops_note": "causal algorithmic: 4 x 128 x q_heads x sum(position + 1) "
                                       "(the reference-order mode computes Q K^T a second time for the "
                                       "row sums; not counted); timed over the whole step"},
            "context": {"torch_sdpa_masked_ms": sdpa_ms,
                        "flash_order": {"ms_per_step": other_ms["flash"],
                                        "tflops": flops / (other_ms["flash"] / 1e3) / 1e12,
                                        "frac": flops / (other_ms["flash"] / 1e3) / 1e12 / peak,
                                        "note": "einsum roundings, unnormalized P rounded, one launch"},
                        "fused_logits": {"ms_per_step": other_ms["fused"],
                                         "tflops": flops / (other_ms["fused"] / 1e3) / 1e12,
                                         "frac": flops / (other_ms["fused"] / 1e3) / 1e12 / peak,
                                         "note": "fp32 logits (the reference's fused NPU attention); "
                                                 "value above keeps the einsum path's roundings and order"}},
            "device_error": int(error.item()), "clocks": clocks.summary(), "cpu_baseline": cpu,
        }), flush=True)


def attention_cpu_sample(positions, query, key, value, scale, budget_s: float = 15.0) -> dict:
    """The oracle's restatement of the reference einsum path on the host, over
    the last query rows until about ``budget_s`` of CPU work."""
    import oracle

    q = query.float().cpu().numpy()
    k = key.float().cpu().numpy()
    v = value.float().cpu().numpy()
    done, t0 = 0, time.perf_counter()
    step = 8
    while time.perf_counter() - t0 < budget_s and done < positions.size:
        rows = slice(positions.size - done - step, positions.size - done)
        limit = int(positions[rows].max()) + 1
        oracle.blend_attention(q[rows], k[:limit], v[:limit], positions[rows], scale, oracle.BF16)
        done += step
    elapsed = time.perf_counter() - t0
    try:
        from threadpoolctl import threadpool_info

        cores = max([int(info.get("num_threads", 1)) for info in threadpool_info()] + [1])
    except ImportError:
        cores = 1
    return {"value": done / elapsed, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"the last {done} query rows, keys up to their positions (numpy oracle; "
                      f"BLAS products on {cores} threads)"}


def attention_reference(args) -> None:
    """--impl reference for config 6: the reference's einsum attention restated
    by the oracle, timed on the host; each step a bounded sample of rows."""
    positions, query, key, value = attention_inputs(1, 0, torch.device("cpu"))
    times = []
    sample = None
    for i in range(args.warmup + args.steps):
        s = attention_cpu_sample(positions, query, key, value, 128 ** -0.5, budget_s=2.0)
        if i >= args.warmup:
            times.append(s["value"])
            sample = s
    value_ = float(np.median(times))
    print(json.dumps({
        "impl": "reference", "metric": "blend-attention query tokens/s (one layer, TP-sharded heads)",
        "value": value_, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16)",
        "config": {"workload": ATTENTION_CONFIG["name"]},
        "cpu_baseline": {**sample, "value": value_},
        "e2e": {"value": value_, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def store_connector(cfg: dict, world: int, rank: int, device):
    """A producer-only ``CacheBlendConnectorV1`` worker built the way vLLM builds it."""
    from types import SimpleNamespace

    from cacheblend_b200.connector import CacheBlendConnectorV1
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole

    transfer = SimpleNamespace(
        engine_id=f"bench-store-{rank}", kv_role="kv_producer", kv_connector="CacheBlendConnectorV1",
        kv_load_failure_policy="fail",
        kv_connector_extra_config={"chunk_size": cfg["chunk"], "local_cpu_gb": cfg["local_cpu_gb"],
                                   "max_inflight_store_batches": cfg["inflight"],
                                   "store_workers": cfg["workers"], "strict_version_check": False})
    vllm_config = SimpleNamespace(
        kv_transfer_config=transfer, cache_config=SimpleNamespace(block_size=cfg["block_size"]),
        parallel_config=SimpleNamespace(tensor_parallel_size=world, pipeline_parallel_size=1),
        model_config=SimpleNamespace(model="Qwen/Qwen3-8B", revision="", dtype="bfloat16"))
    connector = CacheBlendConnectorV1(vllm_config, KVConnectorRole.WORKER)
    heads = cfg["kv_heads"] // world
    pool = cfg["requests"] * cfg["tokens"] // cfg["block_size"]
    gen = torch.Generator(device=device).manual_seed(50 + rank)
    caches = {}
    for layer in range(cfg["layers"]):
        kv = torch.empty(2, pool, cfg["block_size"], heads, cfg["head_dim"], dtype=torch.bfloat16, device=device)
        kv.normal_(generator=gen)
        caches[f"model.layers.{layer}.self_attn.attn"] = kv
    connector.register_kv_caches(caches)
    return connector, caches, heads


def store_metadata(cfg: dict, step: int, rng_tokens: np.ndarray, blocks: np.ndarray):
    """64 prefilled requests; token ids shift per step so every step stores new chunks."""
    from cacheblend_b200.connector import CacheBlendConnectorMetadata, RequestMetadata, _slot_mapping

    meta = CacheBlendConnectorMetadata()
    per_req = cfg["tokens"] // cfg["block_size"]
    for r in range(cfg["requests"]):
        tokens = ((rng_tokens[r] + 7919 * step) % 151_936).tolist()
        slots = _slot_mapping(blocks[r * per_req : (r + 1) * per_req].tolist(), cfg["block_size"], cfg["tokens"])
        meta.requests.append(RequestMetadata(f"s{step}-r{r}", tokens, slots, None, True, cfg["tokens"]))
    return meta


def store_step(connector, caches: dict, meta) -> None:
    """One forward's Store path: every layer's save_kv_layer, then wait_for_save."""
    connector.bind_connector_metadata(meta)
    for name, kv in caches.items():
        connector.save_kv_layer(name, kv, None)
    connector.wait_for_save()
    connector.get_finished({request.request_id for request in meta.requests})


def store_gather_replay(cfg: dict, caches: dict, meta, launches: int = 288) -> tuple[float, int]:
    """Device time (us) and K+V bytes moved (read + written) of one Store gather launch
    with its stream kept busy.

    Inside the steps the Store stream idles while the host enqueues each batch, so
    events around a gather also hold that host time.  This replays batches of the
    step's shape (one request's 32 chunks of one layer, the step's slot mappings)
    back to back, cycling layers and requests so that no launch reads what an
    earlier one left in L2."""
    from cacheblend_b200.kv_layout import describe_paged, device_slots, gather_chunk_major

    layers = list(caches.values())
    paged = [describe_paged(kv, cfg["block_size"]) for kv in layers]
    slots = [device_slots(request.slot_mapping[: cfg["tokens"]], paged[0], cfg["block_size"])
             for request in meta.requests]
    staging = torch.empty(cfg["tokens"] // cfg["chunk"], 2, cfg["chunk"], *layers[0].shape[3:],
                          dtype=layers[0].dtype, device=layers[0].device)
    stream = torch.cuda.Stream(device=layers[0].device)

    def launch(i: int) -> None:
        gather_chunk_major(paged[i % len(paged)], slots[i % len(slots)], staging, stream=stream)

    with torch.cuda.stream(stream):
        for i in range(8):
            launch(i)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(launches):
            launch(i)
        end.record(stream)
    stream.synchronize()
    return start.elapsed_time(end) / launches * 1e3, 2 * staging.numel() * staging.element_size()


def store_cpu_sample(cfg: dict, heads: int, threads: int) -> dict:
    """Oracle gather of 4 requests x 1 layer into host memory, extrapolated."""
    import oracle

    rng = np.random.default_rng(5)
    reqs, bs = 4, cfg["block_size"]
    pool = reqs * cfg["tokens"] // bs
    k = rng.integers(0, 1 << 16, size=(pool, bs, heads, cfg["head_dim"]), dtype=np.uint16) & 0xBFFF
    v = rng.integers(0, 1 << 16, size=k.shape, dtype=np.uint16) & 0xBFFF
    slots = (rng.permutation(pool)[:, None] * bs + np.arange(bs)[None, :]).reshape(-1)
    per = cfg["tokens"]
    t0 = time.perf_counter()
    for r in range(reqs):
        oracle.paged_gather(k, v, slots[r * per : (r + 1) * per], bs, threads)
    dt = time.perf_counter() - t0
    step_s = dt / reqs * cfg["requests"] * cfg["layers"]
    return {"value": cfg["requests"] * cfg["tokens"] / step_s, "step_s": step_s}


def store_reference(args, world: int) -> None:
    import oracle

    cfg = STORE_CONFIG
    threads = oracle.threads(0)
    heads = cfg["kv_heads"] // world
    for _ in range(args.warmup):
        store_cpu_sample(cfg, heads, threads)
    samples = [store_cpu_sample(cfg, heads, threads) for _ in range(args.steps)]
    value = statistics.median(x["value"] for x in samples)
    print(json.dumps({
        "impl": "reference", "metric": "stored prompt tokens/s (all layers: gather + D2H + LRU publication)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.median(x["step_s"] for x in samples) * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": cfg["name"], "parallelism": f"tp{world}"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": "oracle gather of 4 requests x 1 layer, extrapolated to 64 x 36"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def freeze_gc_heap() -> None:
    """vLLM's own startup freeze when it is importable, else the same three collections
    and ``gc.freeze``."""
    try:
        from vllm.utils.gc_utils import freeze_gc_heap as vllm_freeze
    except ImportError:
        gc.collect(0)
        gc.collect(1)
        gc.collect(2)
        gc.freeze()
    else:
        vllm_freeze()


class GcPauses:
    """Collections (count, total and longest pause per generation) while entered."""

    def __init__(self):
        self.pauses: list[tuple[int, float]] = []
        self._start = 0.0

    def _callback(self, phase: str, info: dict) -> None:
        if phase == "start":
            self._start = time.perf_counter()
        else:
            self.pauses.append((info["generation"], (time.perf_counter() - self._start) * 1e3))

    def __enter__(self):
        gc.callbacks.append(self._callback)
        return self

    def __exit__(self, *exc) -> None:
        gc.callbacks.remove(self._callback)

    def summary(self) -> dict:
        out = {}
        for generation in (0, 1, 2):
            ms = [t for g, t in self.pauses if g == generation]
            out[f"gen{generation}"] = {"count": len(ms), "total_ms": round(sum(ms), 2),
                                       "max_ms": round(max(ms), 2) if ms else 0.0}
        return out


def store_bench(args, world: int, rank: int, local: int, steps: int, cpu_on: bool) -> dict | None:
    """Config 5: Store path (gather complete chunks -> D2H -> LRU publication) for 36 layers."""
    cfg = STORE_CONFIG
    device = torch.device("cuda", local)
    connector, caches, heads = store_connector(cfg, world, rank, device)
    if args.store_no_arena:  # per-batch pinned buffers published as views (A/B study)
        connector._store.arena = None
    rng = np.random.default_rng(9)
    rng_tokens = rng.integers(0, 151_936, size=(cfg["requests"], cfg["tokens"]), dtype=np.int64)
    blocks = rng.permutation(cfg["requests"] * cfg["tokens"] // cfg["block_size"])
    metas = [store_metadata(cfg, step, rng_tokens, blocks) for step in range(max(args.warmup, 3) + steps)]
    # the serving process freezes its startup heap before taking requests
    # (vllm/v1/engine/core.py: freeze_gc_heap after init), so a full collection
    # walks only what serving allocated; the pauses inside the timed steps are reported
    freeze_gc_heap()
    gc_pauses = GcPauses()
    row_bytes = heads * cfg["head_dim"] * 2
    step_tokens = cfg["requests"] * cfg["tokens"]
    offered = step_tokens * cfg["layers"] * 2 * row_bytes
    for step in range(max(args.warmup, 3)):
        store_step(connector, caches, metas[step])
    torch.cuda.synchronize(device)
    pipeline = connector._pipeline
    pipeline.kernel_events = []
    d2h_before = pipeline.d2h_bytes
    barrier(world)
    torch.cuda.synchronize(device)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks, gc_pauses:
        start.record()
        for step in range(steps):
            store_step(connector, caches, metas[max(args.warmup, 3) + step])
        end.record()
        torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, device) / steps
    events = pipeline.kernel_events
    pipeline.kernel_events = None
    d2h = (pipeline.d2h_bytes - d2h_before) // steps  # chunks rejected under pressure are not copied
    in_step_us = sum(b.elapsed_time(e) for b, e, _ in events) / len(events) * 1e3
    replay_launches = 288
    # K+V rows read from the pages and written to the staging
    launch_us, launch_bytes = store_gather_replay(cfg, caches, metas[-1], replay_launches)
    peaks = measured_peaks()
    achieved = launch_bytes / (launch_us / 1e6) / 1e9
    link = host_link_peak(device)
    d2h_gbs = d2h / (ms / 1e3) / 1e9
    traffic = load_traffic().get(f"{cfg['name']}:store_gather:tp{world}")
    store = connector._store
    cpu = None
    if rank == 0 and world == 1 and cpu_on:
        import oracle

        threads = oracle.threads(0)
        sample = store_cpu_sample(cfg, heads, threads)
        cpu = {"value": sample["value"], "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": "oracle gather of 4 requests x 1 layer into host memory, extrapolated to 64 x 36"}
    line = None
    if rank == 0:
        value = step_tokens / (ms / 1e3)
        line = {
            "metric": "stored prompt tokens/s (all layers: gather + D2H + LRU publication)", "value": value,
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": max(args.warmup, 3),
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 pages, new token ids every step)",
            "config": {"workload": cfg["name"], "requests": cfg["requests"], "tokens_per_request": cfg["tokens"],
                       "layers": cfg["layers"], "kv_heads_per_rank": heads, "lru_gb": cfg["local_cpu_gb"],
                       "inflight_batches": cfg["inflight"], "store_workers": cfg["workers"],
                       "parallelism": f"tp{world}", "l2": "pages 72 GiB, far larger than L2",
                       "gc": "startup heap frozen as vLLM's engine core does (freeze_gc_heap)"},
            "gpu_launches": len(events),
            "roofline": {"bound": "hbm", "kernel": "store_gather", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                         "avg_launch_us": launch_us, "avg_launch_bytes": launch_bytes,
                         "peak_source": peaks["source"],
                         "timing": f"{replay_launches} launches of the step's batch shape back to back "
                                   "after the timed steps; inside the steps the events around a gather "
                                   "also hold the host's enqueue of the batch (the Store stream idles "
                                   "between batches)",
                         "in_step_event_us": in_step_us},
            "host_link": {"d2h_bytes_per_step": d2h, "offered_bytes_per_step": offered, "d2h_gbs": d2h_gbs, "peak_d2h_gbs": link["d2h_gbs"], "frac": d2h_gbs / link["d2h_gbs"],
                          "peak_source": "measured: best single 1 GiB device->pinned copy"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": d2h,
                    "note": "the Store path starts from vLLM pages in HBM and ends in host memory: value is "
                            "already measured through the connector API with the D2H inside"},
            "store": {"committed_entries": store.committed_entries, "bytes": store.current_bytes,
                      "committed_tokens": store.committed_entries * cfg["chunk"],
                      "gc_pauses_in_timed_steps": gc_pauses.summary(),
                      "pinned_arena_bytes": store.arena.pinned_bytes if store.arena is not None else None,
                      "note": "the LRU budget (16 GiB) holds 455 of the 2,048 chunks offered per step; "
                              "with the pinned arena a chunk that cannot get a slot fails closed before "
                              "its D2H, without it every chunk is copied and the surplus fails at "
                              "publication (d2h_bytes_per_step shows which)"},
            "clocks": clocks.summary(), "cpu_baseline": cpu,
        }
    connector.close()
    del connector, caches
    gc.unfreeze()
    return line


def host_link_scan(args, world: int, rank: int, local: int) -> dict | None:
    """Pinned host <-> device copy bandwidth with every rank copying at once (the
    multi-GPU e2e line rests on the box's aggregate host link).  Each rank copies
    a 1 GiB pinned buffer to its GPU and back, ``args.steps`` times, between
    barriers; the aggregate is all ranks' bytes over the slowest rank's time."""
    device = torch.device("cuda", local)
    nbytes = 1 << 30
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host.fill_(1)
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    out = {}
    for name, dst, src in (("h2d", dev, host), ("d2h", host, dev)):
        for _ in range(2):
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize(device)
        barrier(world)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            dst.copy_(src, non_blocking=True)
        end.record()
        torch.cuda.synchronize(device)
        barrier(world)
        mine = start.elapsed_time(end) / 1e3
        slowest = max_over_ranks(mine, world, device)
        out[name] = {"per_rank_gbs": nbytes * args.steps / mine / 1e9,
                     "aggregate_gbs": world * nbytes * args.steps / slowest / 1e9}
    gathered = [None] * world
    if world > 1:
        torch.distributed.all_gather_object(gathered, out)
    else:
        gathered = [out]
    if rank != 0:
        return None
    return {"metric": "pinned host <-> device copy GB/s, all ranks at once", "n_gpus": world,
            "steps": args.steps, "bytes_per_copy": nbytes,
            "h2d_aggregate_gbs": out["h2d"]["aggregate_gbs"], "d2h_aggregate_gbs": out["d2h"]["aggregate_gbs"],
            "per_rank": gathered}


def deviation_bench(args, shape: Shape, world: int, rank: int, local: int, group, steps: int,
                    e2e_on: bool, cpu_on: bool) -> dict | None:
    """Load + K-deviation score/select + commit for one request through every layer
    (configs 1, 2, 4); returns rank 0's line."""
    device = torch.device("cuda", local)
    shard = args.tp_shard if args.tp_shard and world == 1 else world
    wl = Workload(shape, shard, rank, device, host_store=e2e_on)
    path = DevicePath(wl, tp_group=group)
    path_fused = path.fused
    stream = torch.cuda.Stream(device)
    # warm-up (also builds the check-layer fresh K)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            path.step(stream)
    torch.cuda.synchronize(device)

    # ---- per-kernel CUDA-event durations: an eager pass of the same steps
    barrier(world)
    torch.cuda.synchronize(device)
    path.timing = True
    eager_steps = min(steps, 50)
    with torch.cuda.stream(stream):
        for _ in range(eager_steps):
            path.step(stream)
    torch.cuda.synchronize(device)
    path.timing = False
    barrier(world)

    # ---- value: device-resident inputs, CUDA events on the launching stream
    if not args.no_graph:
        path.capture(stream)
        with torch.cuda.stream(stream):
            for _ in range(3):
                path.step(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    torch.cuda.synchronize(device)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            path.step(stream)
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    path.release()
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world, device)
    ms_per_step = elapsed_ms / steps
    span = wl.act
    value = span / (ms_per_step / 1e3)

    # ---- per-kernel durations: eager CUDA events, then graph replays for the per-layer kernels
    kernel_ms = {name: (sum(s.elapsed_time(e) for s, e in evs) / len(evs)) if evs else None
                 for name, evs in path.events.items()}
    eager_ms = dict(kernel_ms)
    if not args.no_graph:
        for name, us in path.kernel_graph_us(stream, sync=lambda: barrier(world)).items():
            kernel_ms[name] = us / 1e3
    totals = {name: (kernel_ms[name] or 0) * len(path.events[name]) for name in kernel_ms}
    dominant = max(totals, key=totals.get)
    alg = algorithmic_bytes(wl)
    peaks = measured_peaks()
    achieved = alg[dominant] / (kernel_ms[dominant] / 1e3) / 1e9
    traffic = load_traffic().get(f"{shape.name}:{dominant}:" + (f"tp{world}" if shard == world
                                                               else f"tp{shard}-shard"))
    roofline = {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                "peak_source": peaks["source"]}
    per_kernel = {name: {"avg_us": None if ms is None else ms * 1e3,
                         "gbs": None if ms is None else alg[name] / (ms / 1e3) / 1e9,
                         "frac": None if ms is None else alg[name] / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                         "eager_event_us": None if eager_ms[name] is None else eager_ms[name] * 1e3,
                         "launches_per_step": len(path.events[name]) // eager_steps}
                  for name, ms in kernel_ms.items()}

    # ---- the step's one collective: the fp32 score all-reduce (NCCL), timed alone
    allreduce = None
    if world > 1:
        for _ in range(5):
            torch.distributed.all_reduce(path.scores, group=group)
        torch.cuda.synchronize(device)
        barrier(world)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(50):
            torch.distributed.all_reduce(path.scores, group=group)
        a1.record()
        torch.cuda.synchronize(device)
        barrier(world)
        us = max_over_ranks(a0.elapsed_time(a1), world, device) * 1e3 / 50
        allreduce = {"avg_us": us, "bytes": path.scores.numel() * 4,
                     "timing": "50 back-to-back NCCL all-reduces of the step's fp32 score vector, max over ranks"}
        if path.peer is None:
            allreduce["share_of_step"] = us / (ms_per_step * 1e3)
        else:
            allreduce["on_step"] = ("no: the select kernel sums the ranks' scores over NVLink peer memory "
                                    "(cb_select_topk_peer); kernels.select includes that exchange")

    # ---- e2e: public API with host buffers (H2D of reused chunks inside the step)
    e2e = None
    if e2e_on:
        wl.peer = path.peer
        e2e = run_e2e(args, wl, device, world, group, span)
        wl.peer = None
    peer_on = path.peer is not None
    protocol = path.peer.protocol if peer_on else None
    path.close()
    del path, wl
    torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and cpu_on:
        import oracle

        cpu = cpu_baseline(shape, oracle.threads(0))
    if rank != 0:
        return None
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16)",
        "config": workload_config(shape, span, shape.kv_heads // shard, world, shard),
        "gpu_launches": (2 * shape.layers + (1 if path_fused else 2)) * steps,
        "launch": "eager, one stream" if args.no_graph else (
            ("cuda-graph" if world == 1 or peer_on else "two cuda-graphs around the NCCL all-reduce")
            + (", loads on a side stream beside the commits" if 2 * shape.kv_heads // shard * 128 < 2048
               else "")),
        "kernel_timing": ("CUDA events around each launch in an eager pass of the same steps"
                          + ("" if args.no_graph else "; avg_us: each kernel's launches of one step replayed "
                             "as a CUDA graph between two events (deviation / select: ten launches over "
                             "four rotating input sets, 512 MiB, so each reads its inputs from HBM)")),
        "roofline": roofline, "kernels": per_kernel, "e2e": e2e, "allreduce": allreduce,
        "score_reduction": None if world == 1 else (
            f"inside the select kernel over NVLink peer memory (cb_select_topk_peer, {protocol} protocol)"
            if peer_on else "NCCL all-reduce between two graphs"),
        "clocks": clocks.summary(), "cpu_baseline": cpu,
    }


def extra_configs(args, local: int) -> dict:
    """Configs 3, 4 and 5 at one GPU with few steps, for the default run's line."""
    out = {}
    gc.collect()
    torch.cuda.empty_cache()
    cpu_on = not args.no_cpu_baseline
    began = time.perf_counter()
    out["3"] = sparse_q_bench(args, 1, 0, local, steps=20, cpu=cpu_on)
    out["4"] = deviation_bench(args, CONFIGS[4], 1, 0, local, None, steps=20, e2e_on=not args.no_e2e,
                               cpu_on=cpu_on)
    gc.collect()
    torch.cuda.empty_cache()
    out["5"] = store_bench(args, 1, 0, local, steps=3, cpu_on=cpu_on)
    for key, line in out.items():
        if line is not None:
            line["config_index"] = int(key)
    out["wall_s"] = time.perf_counter() - began
    return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None,
                        help="timed steps (default 200; 5 for the seconds-long Store step of config 5)")
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--config", type=int, choices=sorted(CONFIGS) + [3, 5, 6], default=2)
    parser.add_argument("--e2e-steps", type=int, default=5)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-extra-configs", action="store_true",
                        help="config 2 at N=1 only: skip the configs 3/4/5 lines added under 'configs'")
    parser.add_argument("--tp-shard", type=int, default=0,
                        help="run one rank's KV-head shard of an N-way TP step on this GPU alone "
                             "(no all-reduce; per-rank kernel study)")
    parser.add_argument("--no-graph", action="store_true",
                        help="time eager launches instead of CUDA-graph replays of the step")
    parser.add_argument("--layers", type=int, default=0,
                        help="override the layer count (small profiling captures only)")
    parser.add_argument("--attention-tokens", type=int, default=0,
                        help="config 6 context length override (small profiling captures only)")
    parser.add_argument("--store-no-arena", action="store_true",
                        help="config 5: per-batch pinned buffers instead of the pinned arena (A/B study)")
    parser.add_argument("--load-mode", choices=["copy", "zerocopy"], default=None,
                        help="host->device mode of the e2e loader (CACHEBLEND_B200_LOAD)")
    parser.add_argument("--host-link", action="store_true",
                        help="measure pinned host<->device bandwidth with every rank copying at once")
    args = parser.parse_args()
    if args.steps is None:
        args.steps = 5 if args.config == 5 else 200
    if args.load_mode:
        os.environ["CACHEBLEND_B200_LOAD"] = args.load_mode
    world, rank, local, group = dist_setup(args)
    line = None
    if args.host_link:
        line = host_link_scan(args, world, rank, local)
    elif args.config == 3:
        if args.impl == "reference":
            if rank == 0:
                sparse_q_reference(args)
        else:
            line = sparse_q_bench(args, world, rank, local, args.steps, not args.no_cpu_baseline)
    elif args.config == 6:
        global ATTENTION_KEYS
        ATTENTION_KEYS = args.attention_tokens
        if args.impl == "reference":
            if rank == 0:
                attention_reference(args)
        else:
            attention_bench(args, world, rank, local)
    elif args.config == 5:
        if args.impl == "reference":
            if rank == 0:
                store_reference(args, world)
        else:
            line = store_bench(args, world, rank, local, args.steps, not args.no_cpu_baseline)
    else:
        shape = CONFIGS[args.config]
        if args.layers:
            from dataclasses import replace

            shape = replace(shape, name=f"{shape.name}-{args.layers}layers", layers=args.layers)
        if args.impl == "reference":
            run_reference(args, shape, world, rank)
        else:
            line = deviation_bench(args, shape, world, rank, local, group, args.steps, not args.no_e2e,
                                   not args.no_cpu_baseline)
            if (line is not None and world == 1 and args.config == 2 and not args.tp_shard
                    and not args.layers and not args.no_extra_configs):
                line["configs"] = extra_configs(args, local)
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
