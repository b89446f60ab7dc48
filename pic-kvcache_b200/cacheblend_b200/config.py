"""``kv_connector_extra_config`` schema of the connector.

The field set, defaults and validation rules are the API contract of
``CacheBlendConfig`` (cacheblend_vllm/config.py:9-92): a deployment's JSON
config must load unchanged, unknown keys are rejected, and scalar
``check_layers`` / ``recompute_ratios`` are promoted to one-element tuples.
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Any

_STRATEGIES = ("kv_deviation", "sparse_q", "compare")


@dataclass(frozen=True, slots=True)
class CacheBlendConfig:
    chunk_size: int = 256
    local_cpu_gb: float = 16.0
    min_retrieve_tokens: int = 256
    min_hit_ratio: float = 0.10
    min_saved_tokens: int = 0
    max_apc_prefix_to_hit_ratio: float = 0.0
    check_layers: tuple[int, ...] = (1,)
    recompute_ratios: tuple[float, ...] = (0.15,)
    selection_strategy: str = "kv_deviation"
    query_score_chunk_size: int = 8
    overflow_blocks: int = 1
    tail_query_tokens: int = 64
    save_decode_cache: bool = False
    tp_global_selection: bool = True
    event_pipeline: bool = True
    fused_segment_copy: bool = True
    cache_attention_mask: bool = True
    lookup_timeout_ms: int = 10_000
    store_workers: int = 1
    max_inflight_store_batches: int = 8
    strict_version_check: bool = True
    ipc_root: str = "/tmp/cacheblend-v1"
    model_scope: str | None = None

    @classmethod
    def from_extra_config(cls, values: dict[str, Any] | None) -> CacheBlendConfig:
        raw = dict(values or {})
        allowed = {item.name for item in fields(cls)}
        extra = sorted(key for key in raw if key not in allowed)
        if extra:
            raise ValueError(f"Unknown CacheBlend config fields: {extra}")
        for name in ("check_layers", "recompute_ratios"):
            if name in raw:
                value = raw[name]
                raw[name] = (value,) if isinstance(value, (int, float)) else tuple(value)
        config = cls(**raw)
        config.validate()
        return config

    def validate(self) -> None:
        checks: list[tuple[bool, str]] = [
            (self.chunk_size > 0, "chunk_size must be positive"),
            (self.local_cpu_gb > 0, "local_cpu_gb must be positive"),
            (
                self.min_retrieve_tokens >= 0 and self.min_saved_tokens >= 0,
                "token thresholds cannot be negative",
            ),
            (0.0 <= self.min_hit_ratio <= 1.0, "min_hit_ratio must be between 0 and 1"),
            (
                self.max_apc_prefix_to_hit_ratio >= 0,
                "max_apc_prefix_to_hit_ratio cannot be negative",
            ),
            (self.lookup_timeout_ms > 0, "lookup_timeout_ms must be positive"),
            (self.store_workers > 0, "store_workers must be positive"),
            (self.max_inflight_store_batches > 0, "max_inflight_store_batches must be positive"),
            (len(self.check_layers) > 0, "at least one check layer is required"),
            (
                len(self.recompute_ratios) in (1, len(self.check_layers)),
                "recompute_ratios must contain one value or one per check layer",
            ),
            (all(layer >= 0 for layer in self.check_layers), "check layer indices cannot be negative"),
            (
                all(0.0 <= ratio <= 1.0 for ratio in self.recompute_ratios),
                "recompute ratios must be between 0 and 1",
            ),
            (
                self.selection_strategy in _STRATEGIES,
                "selection_strategy must be kv_deviation, sparse_q, or compare",
            ),
        ]
        for ok, message in checks:
            if not ok:
                raise ValueError(message)
        query_aware = self.selection_strategy != "kv_deviation"
        if query_aware and len(self.check_layers) != 1:
            raise ValueError("Sparse-Q selection requires exactly one check layer")
        if self.query_score_chunk_size <= 0:
            raise ValueError("query_score_chunk_size must be positive")
        if self.overflow_blocks < 0:
            raise ValueError("overflow_blocks cannot be negative")
        if self.tail_query_tokens < 0:
            raise ValueError("tail_query_tokens cannot be negative")
        if query_aware and self.tail_query_tokens == 0:
            raise ValueError("Sparse-Q selection requires tail_query_tokens > 0")

    @property
    def max_local_cpu_bytes(self) -> int:
        return int(self.local_cpu_gb * (1 << 30))

    def ratio_for_layer(self, layer_id: int | None) -> float:
        """Recompute ratio of a check layer (first ratio for unknown layers)."""
        position = self.check_layers.index(layer_id) if layer_id in self.check_layers else 0
        return self.recompute_ratios[min(len(self.recompute_ratios) - 1, position)]
