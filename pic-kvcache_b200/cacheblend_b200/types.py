"""Blend plan types: the hot path's input format.

Same fields, invariants and dict wire format as cacheblend_vllm/types.py:10-163
(``SegmentId``, ``BlendSegment``, ``BlendPlan``), because plans travel from
the scheduler process to the workers inside connector metadata.  Besides the
mirror API, ``BlendPlan`` exposes the host-side arrays the kernels consume
(token -> segment map, gap mask, old/new positions).
"""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass, field
from typing import Any

import numpy as np


@dataclass(frozen=True, order=True, slots=True)
class SegmentId:
    model_scope: str
    content_hash: int
    source_start: int
    token_count: int

    def __post_init__(self) -> None:
        if not self.model_scope:
            raise ValueError("model_scope cannot be empty")
        if self.source_start < 0 or self.token_count <= 0:
            raise ValueError("invalid source segment")

    def to_dict(self) -> dict[str, Any]:
        return {
            "model_scope": self.model_scope,
            "content_hash": self.content_hash,
            "source_start": self.source_start,
            "token_count": self.token_count,
        }

    @classmethod
    def from_dict(cls, value: dict[str, Any]) -> SegmentId:
        return cls(
            str(value["model_scope"]),
            int(value["content_hash"]),
            int(value["source_start"]),
            int(value["token_count"]),
        )


@dataclass(frozen=True, order=True, slots=True)
class BlendSegment:
    segment_id: SegmentId
    target_start: int

    def __post_init__(self) -> None:
        if self.target_start < 0:
            raise ValueError("target_start cannot be negative")

    @property
    def source_start(self) -> int:
        return self.segment_id.source_start

    @property
    def length(self) -> int:
        return self.segment_id.token_count

    @property
    def target_end(self) -> int:
        return self.target_start + self.length

    def to_dict(self) -> dict[str, Any]:
        return {"segment_id": self.segment_id.to_dict(), "target_start": self.target_start}

    @classmethod
    def from_dict(cls, value: dict[str, Any]) -> BlendSegment:
        return cls(SegmentId.from_dict(value["segment_id"]), int(value["target_start"]))


@dataclass(frozen=True, slots=True)
class BlendPlan:
    apc_prefix_tokens: int
    allocation_end: int
    hit_tokens: int
    segments: tuple[BlendSegment, ...] = field(default_factory=tuple)

    def __post_init__(self) -> None:
        if self.apc_prefix_tokens < 0 or self.allocation_end < self.apc_prefix_tokens:
            raise ValueError("invalid CacheBlend allocation span")
        by_target = tuple(sorted(self.segments, key=lambda seg: seg.target_start))
        cursor = self.apc_prefix_tokens
        covered = 0
        for seg in by_target:
            if seg.target_start < self.apc_prefix_tokens:
                raise ValueError("segments must start after the APC prefix")
            if seg.target_start < cursor:
                raise ValueError("segments cannot overlap")
            if seg.target_end > self.allocation_end:
                raise ValueError("segment exceeds allocation span")
            covered += seg.length
            cursor = seg.target_end
        if covered != self.hit_tokens:
            raise ValueError(f"hit_tokens={self.hit_tokens} does not match segments={covered}")
        if by_target != self.segments:
            raise ValueError("segments must be sorted")

    @classmethod
    def from_segments(cls, apc_prefix_tokens: int, segments: Iterable[BlendSegment]) -> BlendPlan:
        unique = tuple(sorted(set(segments), key=lambda seg: seg.target_start))
        if not unique:
            return cls(apc_prefix_tokens, apc_prefix_tokens, 0, ())
        return cls(
            apc_prefix_tokens,
            max(seg.target_end for seg in unique),
            sum(seg.length for seg in unique),
            unique,
        )

    @property
    def allocation_tokens(self) -> int:
        return self.allocation_end - self.apc_prefix_tokens

    @property
    def gap_tokens(self) -> int:
        return self.allocation_tokens - self.hit_tokens

    def passes_gate(
        self,
        min_retrieve_tokens: int,
        min_hit_ratio: float,
        min_saved_tokens: int,
        max_apc_prefix_to_hit_ratio: float = 0.0,
    ) -> bool:
        if self.hit_tokens < max(min_retrieve_tokens, min_saved_tokens):
            return False
        if self.hit_tokens / max(self.allocation_tokens, 1) < min_hit_ratio:
            return False
        if max_apc_prefix_to_hit_ratio > 0:
            return self.apc_prefix_tokens / max(self.hit_tokens, 1) <= max_apc_prefix_to_hit_ratio
        return True

    def to_dict(self) -> dict[str, Any]:
        return {
            "apc_prefix_tokens": self.apc_prefix_tokens,
            "allocation_end": self.allocation_end,
            "hit_tokens": self.hit_tokens,
            "segments": [seg.to_dict() for seg in self.segments],
        }

    @classmethod
    def from_dict(cls, value: dict[str, Any]) -> BlendPlan:
        return cls(
            int(value["apc_prefix_tokens"]),
            int(value["allocation_end"]),
            int(value["hit_tokens"]),
            tuple(BlendSegment.from_dict(seg) for seg in value.get("segments", [])),
        )

    # ---- host arrays consumed by the kernels --------------------------------

    def token_segment_map(self) -> np.ndarray:
        """int32[allocation_end]: segment index per token, -1 for gaps/prefix."""
        mapping = np.full(self.allocation_end, -1, dtype=np.int32)
        for index, seg in enumerate(self.segments):
            mapping[seg.target_start : seg.target_end] = index
        return mapping

    def gap_mask(self) -> np.ndarray:
        """bool[allocation_end]: True for tokens no segment covers, after the prefix."""
        mask = np.ones(self.allocation_end, dtype=np.bool_)
        mask[: self.apc_prefix_tokens] = False
        for seg in self.segments:
            mask[seg.target_start : seg.target_end] = False
        return mask

    def hit_positions(self) -> tuple[np.ndarray, np.ndarray]:
        """(old, new) int64 token positions of every hit token, in segment order."""
        if not self.segments:
            empty = np.zeros(0, dtype=np.int64)
            return empty, empty.copy()
        old = np.concatenate(
            [np.arange(seg.source_start, seg.source_start + seg.length) for seg in self.segments]
        )
        new = np.concatenate([np.arange(seg.target_start, seg.target_end) for seg in self.segments])
        return old.astype(np.int64), new.astype(np.int64)
