"""Layerwise side executor: drives one blend request through the local Qwen3
layers and hands the CacheBlend work to the sm_100a seams.

Behaviour kept from Qwen3BlendExecutor (cacheblend_vllm/ascend.py:410-846):
per layer the loader's staging ([2, allocation_end, H, D], old K/V) is taken,
the rows still being computed are projected with the model's own modules
(input norm, qkv, q/k norm, RoPE), check layers score and prune them, the rows'
fresh K/V overwrite the staging, the rows attend over the whole staging, then
o_proj, post-attention norm and MLP run and the staging is committed back to
vLLM's pages.  Strategies at a check layer:

* ``kv_deviation`` -- prune before the layer's attention by K-deviation
  (ascend.py:534-543, 600-609);
* ``sparse_q`` -- score the gap queries against the staged keys with the fresh
  keys written in place, attend with every row, prune after the MLP
  (ascend.py:545-566, 618-630);
* ``compare`` -- prune by K-deviation and trace the overlap of both selections
  (ascend.py:568-577).

How it is organised here: a layer is four stages over a ``_Rows`` bundle
(``_project`` -> ``_choose`` -> ``_stage_and_attend`` -> ``_feed_forward``),
each stage a call into vLLM's modules or one ``cacheblend_b200`` entry point
(``kv_deviation``, ``sparse_q_scores``, ``select_tokens``, ``blend_attention``).
The gap mask stays on the host, and the absolute rows are mirrored there while
they are a plain range (before any pruning), so the check layer's masks and
budgets need no device read.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import torch

from .attention import attention_supported, attention_workspace_bytes, blend_attention
from .config import CacheBlendConfig
from .rope import validate_rope_support
from .peer_exchange import MAX_PEERS, MAX_TOKENS, PeerExchangeUnavailable, PeerScoreExchange
from .selection import (deviation_select, kv_deviation, select_tokens, selection_overlap,
                        sparse_q_scores, tp_world_size)
from .trace import PipelineTracer
from .types import BlendPlan

# CACHEBLEND_B200_ATTENTION=fused: fp32 logits like the reference's fused NPU attention
# (ascend.py:814-830); =flash: the einsum path's roundings with flash-order normalization
# (one launch); default: the einsum path's roundings in its own order, which is what the
# reference computes on a CUDA device.
_ATTENTION_MODE = os.environ.get("CACHEBLEND_B200_ATTENTION", "").lower() or "reference"
if _ATTENTION_MODE not in ("reference", "flash", "fused"):
    raise ValueError(f"CACHEBLEND_B200_ATTENTION must be reference, flash or fused, not {_ATTENTION_MODE!r}")

# CACHEBLEND_B200_FUSED_SELECT=1: K-deviation and selection of a one-rank check layer as one
# launch (cb_kv_deviation_select) instead of two (measured slower on B200 so far: off by default)
_FUSED_SELECT = os.environ.get("CACHEBLEND_B200_FUSED_SELECT", "") == "1"
# With TP the score all-reduce runs inside the select kernel over NVLink peer memory
# (cb_select_topk_peer); CACHEBLEND_B200_PEER_SELECT=0 puts vLLM's NCCL all-reduce back.
_PEER_SELECT = os.environ.get("CACHEBLEND_B200_PEER_SELECT", "1") != "0"

_EMBEDDING_HOOKS = ("get_input_embeddings", "embed_input_ids")


def _token_embeddings(model, token_ids: torch.Tensor) -> torch.Tensor:
    """Embeddings of ``token_ids`` through whichever hook this vLLM model exposes."""
    getter = getattr(model, "get_input_embeddings", None)
    if getter is not None:
        table = getter()
        if callable(table):
            return table(token_ids)
    embed = getattr(model, "embed_input_ids", None)
    if embed is not None:
        return embed(token_ids)
    inner = getattr(model.model, "embed_tokens", None)
    if inner is not None:
        return inner(token_ids)
    raise AttributeError(f"{type(model).__name__} exposes none of {_EMBEDDING_HOOKS} or embed_tokens")


def _tensor_parallel_group():
    """vLLM's TP group coordinator, or None outside a vLLM worker."""
    try:
        from vllm.distributed.parallel_state import get_tp_group

        return get_tp_group()
    except (AssertionError, ImportError):
        return None


@dataclass(slots=True)
class BlendExecutionState:
    """Per-request state carried from layer to layer.

    ``important_indices``: rows (relative to ``compute_start``) still computed,
    None while every row is; ``positions``: their token positions;
    ``gap_mask``: host bool [allocation_end]; ``attention_mask``: cached mask
    of the torch attention fallback."""

    compute_start: int
    positions: torch.Tensor
    gap_mask: np.ndarray
    important_indices: torch.Tensor | None = None
    attention_mask: torch.Tensor | None = None


@dataclass(slots=True)
class _Rows:
    """One layer's tensors for the rows it computes, row-aligned."""

    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    residual: torch.Tensor
    relative: torch.Tensor  # row ids relative to compute_start (device, int64)
    positions: torch.Tensor
    absolute: torch.Tensor  # staging rows = compute_start + relative
    absolute_host: np.ndarray | None  # host mirror when known without a device read

    def keep(self, chosen: torch.Tensor) -> _Rows:
        return _Rows(self.q[chosen], self.k[chosen], self.v[chosen], self.residual[chosen],
                     self.relative[chosen], self.positions[chosen], self.absolute[chosen], None)

    def host_absolute(self) -> np.ndarray:
        if self.absolute_host is None:  # rows pruned by an earlier check layer: one read
            self.absolute_host = self.absolute.detach().to("cpu").numpy()
        return self.absolute_host

    def span(self) -> slice | None:
        """The staging rows as one slice when they are a plain ascending range."""
        host = self.absolute_host
        if host is None or host.size == 0:
            return None
        first = int(host[0])
        return slice(first, first + host.size) if int(host[-1]) == first + host.size - 1 else None


@dataclass(slots=True)
class _Choice:
    """What a check layer decided: rows to keep before attention / after the MLP."""

    before_attention: torch.Tensor | None = None
    after_feed_forward: torch.Tensor | None = None
    stats: dict | None = None


def _overwrite_rows(plane: torch.Tensor, rows: _Rows, values: torch.Tensor) -> None:
    """plane[absolute rows] = values (a plain copy when the rows are a range)."""
    where = rows.span()
    if where is not None:
        plane[where].copy_(values)
    else:
        plane[rows.absolute] = values


class Qwen3BlendExecutor:
    """Runs the blend span through this rank's decoder layers, one layer at a time."""

    def __init__(self, model, config: CacheBlendConfig, block_size: int):
        if block_size <= 0:
            raise ValueError("vLLM KV cache block_size must be positive")
        inner = model.model
        layers = list(inner.layers[inner.start_layer : inner.end_layer])
        if not layers:
            raise RuntimeError("Qwen3 model has no local decoder layers")
        if max(config.check_layers) >= len(layers):
            raise ValueError(
                "CacheBlend check layer exceeds the local Qwen3 layer range: "
                f"check_layers={config.check_layers}, layers={len(layers)}"
            )
        validate_rope_support(model, layers[0].self_attn.rotary_emb)
        self.model = model
        self.config = config
        self.block_size = block_size
        self.layers = layers
        self.tp_group = _tensor_parallel_group()
        self._peer: PeerScoreExchange | None = None  # made by the first TP selection
        self._peer_unavailable = False

    def _peer_exchange(self, tokens: int, device: torch.device) -> PeerScoreExchange | None:
        """The TP group's peer-memory score exchange when this selection can use it.  Every
        rank reaches the same decision (same request, same token count), and the exchange
        is created collectively by the first selection that needs it."""
        world = tp_world_size(self.tp_group)
        if not (_PEER_SELECT and self.config.tp_global_selection and 1 < world <= MAX_PEERS
                and tokens <= MAX_TOKENS and device.type == "cuda") or self._peer_unavailable:
            return None
        if self._peer is None:
            try:
                self._peer = PeerScoreExchange(self.tp_group, MAX_TOKENS, device)
            except PeerExchangeUnavailable:
                self._peer_unavailable = True  # every rank: vLLM's all-reduce from now on
                return None
        return self._peer

    # ------------------------------------------------------------------ request
    def run(self, request_id: str, tokens: list[int], plan: BlendPlan, loader) -> None:
        """Layerwise pass over ``[apc_prefix, allocation_end)`` with the loader's
        prefetch(l + 1) overlapping layer l (ascend.py:433-485)."""
        first, end = plan.apc_prefix_tokens, plan.allocation_end
        if end <= first:
            return
        cache = loader.kv_caches[0]
        device = (cache if isinstance(cache, torch.Tensor) else cache[0]).device
        hidden = _token_embeddings(self.model, torch.tensor(tokens[first:end], dtype=torch.long,
                                                              device=device))
        state = BlendExecutionState(first, torch.arange(first, end, device=device), plan.gap_mask())
        residual = None
        depth = len(self.layers)
        tracer = loader.tracer
        loader.prefetch(0, self.layers[0].self_attn.rotary_emb)
        for index in range(depth):
            staging = loader.get(index)
            if index + 1 < depth:
                loader.prefetch(index + 1, self.layers[index + 1].self_attn.rotary_emb)
            hidden, residual, state, staging = self._compute_layer(
                index, self.layers[index], hidden, residual, state, staging,
                request_id=request_id, tracer=tracer)
            _emit(tracer, "layer_compute_enqueued", request_id, layer_id=index,
                  computed_tokens=int(hidden.shape[0]), check_layer=index in self.config.check_layers)
            loader.commit(index, staging)

    # -------------------------------------------------------------------- layer
    def _compute_layer(self, layer_id: int, layer, hidden_states: torch.Tensor,
                       residual: torch.Tensor | None, state: BlendExecutionState,
                       old_kv: torch.Tensor, request_id: str | None = None,
                       tracer: PipelineTracer | None = None):
        """One decoder layer over the computed rows; returns (hidden, residual, state, staging)."""
        rows = self._project(layer, hidden_states, residual, state)
        choice = self._choose(layer_id, layer, rows, state, old_kv, request_id, tracer)
        if choice.before_attention is not None:
            rows = rows.keep(choice.before_attention)
            _narrow(state, rows.relative, rows.positions)
        attended = self._stage_and_attend(layer, rows, old_kv, state)
        hidden, residual = self._feed_forward(layer, attended, rows.residual)
        if choice.after_feed_forward is not None:
            chosen = choice.after_feed_forward
            hidden, residual = hidden[chosen], residual[chosen]
            _narrow(state, rows.relative[chosen], rows.positions[chosen])
            _emit(tracer, "selection_finished", request_id, layer_id=layer_id, strategy="sparse_q",
                  selected_tokens=int(chosen.numel()), **(choice.stats or {}))
        return hidden, residual, state, old_kv

    def _project(self, layer, hidden: torch.Tensor, residual: torch.Tensor | None,
                 state: BlendExecutionState) -> _Rows:
        """Input norm (fused with the residual add after the first layer), qkv
        projection, per-head q/k norm and RoPE at the rows' positions."""
        if residual is None:
            residual, hidden = hidden, layer.input_layernorm(hidden)
        else:
            hidden, residual = layer.input_layernorm(hidden, residual)
        attn = layer.self_attn
        qkv, _ = attn.qkv_proj(hidden)
        q, k, v = qkv.split([attn.q_size, attn.kv_size, attn.kv_size], dim=-1)
        width = attn.head_dim
        q = attn.q_norm(q.reshape(q.shape[0], -1, width)).reshape(q.shape)
        k = attn.k_norm(k.reshape(k.shape[0], -1, width)).reshape(k.shape)
        q, k = attn.rotary_emb(state.positions, q, k)
        count = q.shape[0]
        if state.important_indices is None:
            relative = torch.arange(count, device=q.device)
            host = np.arange(state.compute_start, state.compute_start + count, dtype=np.int64)
        else:
            relative, host = state.important_indices, None
        return _Rows(q, k, v, residual, relative, state.positions, state.compute_start + relative, host)

    def _choose(self, layer_id: int, layer, rows: _Rows, state: BlendExecutionState,
                staging: torch.Tensor, request_id, tracer) -> _Choice:
        """Scores and selections of a check layer (nothing elsewhere)."""
        if layer_id not in self.config.check_layers:
            return _Choice()
        strategy = self.config.selection_strategy
        gaps = state.gap_mask[rows.host_absolute()]
        cached_k = staging[0].view(staging.shape[1], -1)  # a view: sparse_q writes through it
        choice = _Choice()
        by_deviation = by_query = None
        if strategy in ("kv_deviation", "compare"):
            ratio = self.config.ratio_for_layer(layer_id)
            if _FUSED_SELECT and not (self.config.tp_global_selection and tp_world_size(self.tp_group) > 1):
                # this rank's scores alone: score and select in one launch
                by_deviation, _ = deviation_select(rows.k, cached_k, gaps, ratio, rows.absolute)
            else:
                deviation = kv_deviation(rows.k, cached_k, rows.absolute)
                by_deviation = self._select(deviation, gaps, layer_id)  # all-reduce (TP), then select
            choice.before_attention = by_deviation
        if strategy in ("sparse_q", "compare"):
            attn = layer.self_attn.attn
            # the boundary score sees the fresh keys of the computed rows; in
            # sparse_q mode they are written into the staging itself (the
            # write-back below stores the same values), in compare mode into a copy
            keys = cached_k if strategy == "sparse_q" else cached_k.clone()
            _overwrite_rows(keys, rows, rows.k)
            heads, kv_heads, head = int(attn.num_heads), int(attn.num_kv_heads), int(attn.head_size)
            scores, forced, stats = sparse_q_scores(
                rows.q.view(-1, heads, head), keys.view(-1, kv_heads, head), rows.host_absolute(),
                gaps, float(attn.impl.scale), self.block_size, self.config.overflow_blocks,
                self.config.tail_query_tokens)
            by_query = self._select(scores, gaps, layer_id, forced_mask=forced)
            choice.stats = stats
            if strategy == "sparse_q":
                choice.after_feed_forward = by_query
        if strategy == "compare" and tracer is not None and tracer.enabled:
            overlap, union = selection_overlap(by_deviation, by_query)
            _emit(tracer, "selection_compared", request_id, layer_id=layer_id,
                  deviation_tokens=by_deviation.numel(), sparse_q_tokens=by_query.numel(),
                  overlap_tokens=overlap, jaccard=overlap / max(union, 1), **choice.stats)
        return choice

    def _select(self, scores: torch.Tensor, gaps: np.ndarray, layer_id: int,
                forced_mask=None) -> torch.Tensor:
        """TP-summed, budgeted top-k united with the gap (and forced) rows (ascend.py:757-796)."""
        return select_tokens(scores, gaps, self.config.ratio_for_layer(layer_id), forced_mask,
                             tp_group=self.tp_group, global_selection=self.config.tp_global_selection,
                             peer_exchange=self._peer_exchange(scores.numel(), scores.device))

    def _stage_and_attend(self, layer, rows: _Rows, staging: torch.Tensor,
                          state: BlendExecutionState) -> torch.Tensor:
        """Fresh K/V of the computed rows into the staging, then their attention over it."""
        plane_rows = staging.shape[1]
        _overwrite_rows(staging[0].view(plane_rows, -1), rows, rows.k)
        _overwrite_rows(staging[1].view(plane_rows, -1), rows, rows.v)
        attn = layer.self_attn.attn
        heads, kv_heads, head = int(attn.num_heads), int(attn.num_kv_heads), int(attn.head_size)
        out = self._attend(rows.q.view(-1, heads, head), staging[0].view(-1, kv_heads, head),
                           staging[1].view(-1, kv_heads, head), rows.absolute, float(attn.impl.scale),
                           state)
        return out.reshape(-1, heads * head)

    def _feed_forward(self, layer, attended: torch.Tensor, residual: torch.Tensor):
        hidden, _ = layer.self_attn.o_proj(attended)
        hidden, residual = layer.post_attention_layernorm(hidden, residual)
        return layer.mlp(hidden), residual

    def _attend(self, query, key, value, positions, scale: float, state: BlendExecutionState):
        """Causal attention of the computed queries over the whole staging
        (ascend.py:798-846): the tcgen05 kernel for head size 128 in bf16/fp16
        with query groups dividing 128 (every Qwen3 shape), torch SDPA with the
        same mask otherwise."""
        if query.device.type == "cuda" and attention_supported(query, key):
            need = attention_workspace_bytes(query.shape[0], key.shape[0], query.shape[1], key.shape[1],
                                             query.shape[2], query.dtype)
            scratch = getattr(self, "_attention_scratch", None)
            if scratch is None or scratch.numel() < need or scratch.device != query.device:
                scratch = torch.empty(need, dtype=torch.uint8, device=query.device)
                self._attention_scratch = scratch
            return blend_attention(query, key, value, positions, scale, workspace=scratch,
                                   exact_rounding="reference" if scale <= 0 and _ATTENTION_MODE == "fused"
                                   else _ATTENTION_MODE)
        reuse = self.config.cache_attention_mask and state.important_indices is not None
        visible = state.attention_mask if reuse else None
        if visible is None:
            visible = positions[:, None] >= torch.arange(key.shape[0], device=query.device)[None, :]
            if reuse:
                state.attention_mask = visible
        out = torch.nn.functional.scaled_dot_product_attention(
            query.transpose(0, 1)[None], key.transpose(0, 1)[None], value.transpose(0, 1)[None],
            attn_mask=visible[None, None], scale=scale, enable_gqa=query.shape[1] != key.shape[1])
        return out[0].transpose(0, 1)


def _narrow(state: BlendExecutionState, relative: torch.Tensor, positions: torch.Tensor) -> None:
    state.important_indices = relative
    state.positions = positions
    state.attention_mask = None


def _emit(tracer: PipelineTracer | None, event: str, request_id, **fields) -> None:
    if tracer is not None and tracer.enabled:
        tracer.emit(event, request_id=request_id, **fields)
