"""Layerwise side executor for Qwen3 with the hot-path seams on B200 kernels.

Control flow follows Qwen3BlendExecutor (cacheblend_vllm/ascend.py:410-846):
embed the span, then per layer get the loader's staging (old K/V), run the
model's norms / qkv / q-k norm + RoPE, at check layers score and select the
tokens to recompute, prune, write the fresh K/V into the staging, attend,
o_proj + MLP, and commit the staging back into vLLM's pages.  The model math
is vLLM's own modules; the CacheBlend work -- staging load, K-deviation,
Sparse-Q scoring, top-k selection (with the TP all-reduce) and the commit --
runs on the sm_100a kernels through ``cacheblend_b200``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

import os

from .attention import attention_supported, attention_workspace_bytes, blend_attention
from .config import CacheBlendConfig
from .loader import PagedBlendLoader
from .rope import validate_rope_support
from .selection import kv_deviation, select_tokens, selection_overlap, sparse_q_scores
from .trace import PipelineTracer
from .types import BlendPlan


# CACHEBLEND_B200_ATTENTION=fused: fp32 logits like the reference's fused NPU attention
# (ascend.py:814-830) instead of the einsum path's element-type roundings (the default,
# which is what the reference runs on a CUDA device).
_FUSED_ATTENTION = os.environ.get("CACHEBLEND_B200_ATTENTION", "").lower() == "fused"


def _embed(model, input_ids: torch.Tensor) -> torch.Tensor:
    if hasattr(model, "get_input_embeddings"):
        embeddings = model.get_input_embeddings()
        if callable(embeddings):
            return embeddings(input_ids)
    if hasattr(model, "embed_input_ids"):
        return model.embed_input_ids(input_ids)
    if hasattr(model.model, "embed_tokens"):
        return model.model.embed_tokens(input_ids)
    raise AttributeError(f"{type(model).__name__} has no supported embedding API")


@dataclass(slots=True)
class BlendExecutionState:
    compute_start: int
    positions: torch.Tensor
    gap_mask: np.ndarray  # host copy: [allocation_end]
    important_indices: torch.Tensor | None = None
    attention_mask: torch.Tensor | None = None


class Qwen3BlendExecutor:
    def __init__(self, model, config: CacheBlendConfig, block_size: int):
        self.model = model
        self.config = config
        if block_size <= 0:
            raise ValueError("vLLM KV cache block_size must be positive")
        self.block_size = block_size
        self.layers = list(model.model.layers[model.model.start_layer : model.model.end_layer])
        if not self.layers:
            raise RuntimeError("Qwen3 model has no local decoder layers")
        if max(config.check_layers) >= len(self.layers):
            raise ValueError(
                "CacheBlend check layer exceeds the local Qwen3 layer range: "
                f"check_layers={config.check_layers}, layers={len(self.layers)}"
            )
        validate_rope_support(model, self.layers[0].self_attn.rotary_emb)
        try:
            from vllm.distributed.parallel_state import get_tp_group

            self.tp_group = get_tp_group()
        except (AssertionError, ImportError):
            self.tp_group = None

    # ------------------------------------------------------------------ run
    def run(self, request_id: str, tokens: list[int], plan: BlendPlan, loader: PagedBlendLoader) -> None:
        if plan.allocation_end <= plan.apc_prefix_tokens:
            return
        device = loader.kv_caches[0].device if isinstance(loader.kv_caches[0], torch.Tensor) \
            else loader.kv_caches[0][0].device
        input_ids = torch.tensor(
            tokens[plan.apc_prefix_tokens : plan.allocation_end], dtype=torch.long, device=device
        )
        hidden_states = _embed(self.model, input_ids)
        residual = None
        positions = torch.arange(plan.apc_prefix_tokens, plan.allocation_end, device=device)
        state = BlendExecutionState(plan.apc_prefix_tokens, positions, plan.gap_mask())
        loader.prefetch(0, self.layers[0].self_attn.rotary_emb)
        for layer_id, layer in enumerate(self.layers):
            old_kv = loader.get(layer_id)
            if layer_id + 1 < len(self.layers):
                loader.prefetch(layer_id + 1, self.layers[layer_id + 1].self_attn.rotary_emb)
            hidden_states, residual, state, old_kv = self._compute_layer(
                layer_id, layer, hidden_states, residual, state, old_kv,
                request_id=request_id, tracer=loader.tracer,
            )
            if loader.tracer is not None and loader.tracer.enabled:
                loader.tracer.emit(
                    "layer_compute_enqueued",
                    request_id=request_id,
                    layer_id=layer_id,
                    computed_tokens=int(hidden_states.shape[0]),
                    check_layer=layer_id in self.config.check_layers,
                )
            loader.commit(layer_id, old_kv)

    def _compute_layer(self, layer_id, layer, hidden_states, residual, state, old_kv,
                       request_id=None, tracer: PipelineTracer | None = None):
        if residual is None:
            residual = hidden_states
            hidden_states = layer.input_layernorm(hidden_states)
        else:
            hidden_states, residual = layer.input_layernorm(hidden_states, residual)
        qkv, _ = layer.self_attn.qkv_proj(hidden_states)
        q, k, v = qkv.split(
            [layer.self_attn.q_size, layer.self_attn.kv_size, layer.self_attn.kv_size], dim=-1
        )
        query_indices = (
            torch.arange(q.shape[0], device=q.device)
            if state.important_indices is None
            else state.important_indices
        )
        absolute_indices = state.compute_start + query_indices
        q, k = self._qk_post_process(layer.self_attn, state.positions, q, k)
        flat_old_k = old_kv[0].reshape(old_kv.shape[1], -1)
        flat_old_v = old_kv[1].reshape(old_kv.shape[1], -1)
        check_layer = layer_id in self.config.check_layers
        strategy = self.config.selection_strategy
        deviation_selected = sparse_q_selected = None
        stats: dict = {}
        if check_layer:
            abs_host = absolute_indices.detach().to("cpu").numpy()
            active_gap_mask = state.gap_mask[abs_host]
        if check_layer and strategy in {"kv_deviation", "compare"}:
            scores = kv_deviation(k, flat_old_k, absolute_indices)
            deviation_selected = self._select(scores, active_gap_mask, layer_id)
        if check_layer and strategy in {"sparse_q", "compare"}:
            attn = layer.self_attn.attn
            score_keys = flat_old_k if strategy == "sparse_q" else flat_old_k.clone()
            score_keys[absolute_indices] = k
            scores, forced, stats = self._sparse_q_scores(
                q.view(-1, int(attn.num_heads), int(attn.head_size)),
                score_keys.view(-1, int(attn.num_kv_heads), int(attn.head_size)),
                abs_host,
                active_gap_mask,
                float(attn.impl.scale),
            )
            sparse_q_selected = self._select(scores, active_gap_mask, layer_id, forced_mask=forced)
        if check_layer and strategy == "compare" and tracer is not None and tracer.enabled:
            overlap, union = selection_overlap(deviation_selected, sparse_q_selected)
            tracer.emit("selection_compared", request_id=request_id, layer_id=layer_id,
                        deviation_tokens=deviation_selected.numel(),
                        sparse_q_tokens=sparse_q_selected.numel(), overlap_tokens=overlap,
                        jaccard=overlap / max(union, 1), **stats)
        if check_layer and strategy in {"kv_deviation", "compare"}:
            selected = deviation_selected
            q, k, v = q[selected], k[selected], v[selected]
            residual = residual[selected]
            query_indices = query_indices[selected]
            absolute_indices = state.compute_start + query_indices
            state.important_indices = query_indices
            state.positions = state.positions[selected]
            state.attention_mask = None
        flat_old_k[absolute_indices] = k
        flat_old_v[absolute_indices] = v
        attn = layer.self_attn.attn
        num_heads, num_kv_heads, head_size = int(attn.num_heads), int(attn.num_kv_heads), int(attn.head_size)
        attn_output = self._attention(
            q.view(-1, num_heads, head_size),
            old_kv[0].view(-1, num_kv_heads, head_size),
            old_kv[1].view(-1, num_kv_heads, head_size),
            absolute_indices,
            float(attn.impl.scale),
            state,
        ).reshape(-1, num_heads * head_size)
        hidden_states, _ = layer.self_attn.o_proj(attn_output)
        hidden_states, residual = layer.post_attention_layernorm(hidden_states, residual)
        hidden_states = layer.mlp(hidden_states)
        if check_layer and strategy == "sparse_q":
            hidden_states = hidden_states[sparse_q_selected]
            residual = residual[sparse_q_selected]
            query_indices = query_indices[sparse_q_selected]
            state.important_indices = query_indices
            state.positions = state.positions[sparse_q_selected]
            state.attention_mask = None
            if tracer is not None and tracer.enabled:
                tracer.emit("selection_finished", request_id=request_id, layer_id=layer_id,
                            strategy="sparse_q", selected_tokens=int(sparse_q_selected.numel()), **stats)
        return hidden_states, residual, state, old_kv

    # ------------------------------------------------------------- seams
    def _sparse_q_scores(self, query, key, absolute_indices, gap_mask, scale):
        """Per-active-token Sparse-Q scores, forced mask and stats (ascend.py:638-711)."""
        return sparse_q_scores(
            query, key, absolute_indices, gap_mask, scale, self.block_size,
            self.config.overflow_blocks, self.config.tail_query_tokens,
        )

    def _select(self, scores, gap_mask, layer_id=None, forced_mask=None) -> torch.Tensor:
        """TP-reduced, budgeted top-k union with gaps/forced (ascend.py:757-796)."""
        return select_tokens(
            scores,
            gap_mask,
            self.config.ratio_for_layer(layer_id),
            forced_mask,
            tp_group=self.tp_group,
            global_selection=self.config.tp_global_selection,
        )

    @staticmethod
    def _qk_post_process(attn_layer, positions, q, k):
        q_heads = q.view(*q.shape[:-1], q.shape[-1] // attn_layer.head_dim, attn_layer.head_dim)
        q = attn_layer.q_norm(q_heads).view(q.shape)
        k_heads = k.view(*k.shape[:-1], k.shape[-1] // attn_layer.head_dim, attn_layer.head_dim)
        k = attn_layer.k_norm(k_heads).view(k.shape)
        return attn_layer.rotary_emb(positions, q, k)

    def _attention(self, query, key, value, q_positions, scale, state: BlendExecutionState):
        """Causal attention of the computed queries over the whole staging context
        (ascend.py:798-846).  Head size 128 in bf16 / fp16 with query groups
        dividing 128 (every Qwen3 configuration) runs the tcgen05 kernel; other
        shapes use torch's SDPA with the same mask."""
        if query.device.type == "cuda" and attention_supported(query, key):
            need = attention_workspace_bytes(query.shape[0], key.shape[0], query.shape[1],
                                             key.shape[1], query.shape[2], query.dtype)
            workspace = getattr(self, "_attention_workspace", None)
            if workspace is None or workspace.numel() < need or workspace.device != query.device:
                workspace = torch.empty(need, dtype=torch.uint8, device=query.device)
                self._attention_workspace = workspace
            return blend_attention(query, key, value, q_positions, scale, workspace=workspace,
                                   exact_rounding=not _FUSED_ATTENTION or scale <= 0)
        k_positions = torch.arange(key.shape[0], device=query.device)
        cache = self.config.cache_attention_mask and state.important_indices is not None
        allowed = state.attention_mask if cache else None
        if allowed is None:
            allowed = q_positions[:, None] >= k_positions[None, :]
            if cache:
                state.attention_mask = allowed
        out = torch.nn.functional.scaled_dot_product_attention(
            query.transpose(0, 1)[None],
            key.transpose(0, 1)[None],
            value.transpose(0, 1)[None],
            attn_mask=allowed[None, None],
            scale=scale,
            enable_gqa=query.shape[1] != key.shape[1],
        )
        return out[0].transpose(0, 1)
