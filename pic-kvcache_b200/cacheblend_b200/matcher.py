"""Content fingerprints and the token-range matcher behind the store.

The fingerprint function is part of the store's wire contract: segment ids
(and therefore cache hits across processes) depend on it.  It is the 64-bit
polynomial hash of cacheblend_vllm/hashing.py:18-22 -- base 1,000,003 over
``token + 1``, wrapping modulo 2**64.  Window hashes at every offset are
computed in O(N) here (instead of the reference's O(N x window) sliding
matmul, hashing.py:42-53) from prefix sums in the ring Z/2**64: because the
base is odd it is invertible modulo 2**64, so

    hash(tokens[i:i+W]) = B**(i+W) * (Q[i+W] - Q[i]),  Q[j] = sum_{t<j} v_t * B**-(t+1)

Matching semantics follow TokenRangeMatcher.match (matcher.py:80-125):
leftmost-greedy, non-overlapping, with exact token verification.
"""

from __future__ import annotations

import threading
from collections import defaultdict
from collections.abc import Iterable, Sequence
from dataclasses import dataclass

import numpy as np

from .types import BlendSegment, SegmentId

POLY_BASE = 1_000_003
_MOD = 1 << 64
_BASE_INV = pow(POLY_BASE, -1, _MOD)


def content_hash(tokens: Sequence[int]) -> int:
    """Polynomial fingerprint of one chunk (exact Python integer arithmetic)."""
    value = 0
    for token in tokens:
        value = (value * POLY_BASE + int(token) + 1) % _MOD
    return value


def _powers(base: int, count: int) -> np.ndarray:
    """[base**0, base**1, ..., base**(count-1)] modulo 2**64 as uint64."""
    out = np.empty(count, dtype=np.uint64)
    if count == 0:
        return out
    out[0] = 1
    if count > 1:
        out[1:] = np.uint64(base)
        with np.errstate(over="ignore"):
            np.cumprod(out, out=out)
    return out


def window_hashes(tokens: Sequence[int] | np.ndarray, window: int) -> np.ndarray:
    """uint64 fingerprint of every full window of ``tokens`` (O(N))."""
    if window <= 0:
        raise ValueError("window must be positive")
    values = np.asarray(tokens, dtype=np.int64).astype(np.uint64) + np.uint64(1)
    n = values.shape[0]
    if n < window:
        return np.empty(0, dtype=np.uint64)
    with np.errstate(over="ignore"):
        inv_pows = _powers(_BASE_INV, n + 1)[1:]  # B**-(t+1)
        prefix = np.zeros(n + 1, dtype=np.uint64)
        np.cumsum(values * inv_pows, out=prefix[1:])
        pows = _powers(POLY_BASE, n + 1)
        starts = np.arange(n - window + 1)
        return pows[starts + window] * (prefix[starts + window] - prefix[starts])


def chunk_hashes(chunks: np.ndarray) -> np.ndarray:
    """uint64 fingerprint of each row of ``chunks`` [count, width]: Horner's
    recurrence unrolled to sum_i (t_i + 1) * B**(width-1-i), wrapping mod 2**64."""
    values = np.asarray(chunks, dtype=np.int64).astype(np.uint64) + np.uint64(1)
    with np.errstate(over="ignore"):
        weights = _powers(POLY_BASE, values.shape[1])[::-1]
        return (values * weights).sum(axis=1, dtype=np.uint64)


@dataclass(frozen=True, slots=True)
class FingerprintRecord:
    segment_id: SegmentId
    tokens: tuple[int, ...]


class TokenRangeMatcher:
    """Committed chunk fingerprints, matchable at any token offset."""

    def __init__(self, chunk_size: int):
        if chunk_size <= 0:
            raise ValueError("chunk_size must be positive")
        self.chunk_size = chunk_size
        self._records: dict[SegmentId, FingerprintRecord] = {}
        self._by_hash: dict[tuple[str, int], list[FingerprintRecord]] = defaultdict(list)
        self._hashes: dict[str, set[int]] = defaultdict(set)
        self._lock = threading.RLock()

    def make_record(
        self, model_scope: str, source_start: int, tokens: Sequence[int]
    ) -> FingerprintRecord:
        if len(tokens) != self.chunk_size:
            raise ValueError(
                f"fingerprint requires exactly {self.chunk_size} tokens, got {len(tokens)}"
            )
        chunk = tuple(int(token) for token in tokens)
        return FingerprintRecord(
            SegmentId(model_scope, content_hash(chunk), source_start, len(chunk)), chunk
        )

    def make_records(
        self, model_scope: str, first_start: int, tokens: Sequence[int] | np.ndarray, count: int
    ) -> list[FingerprintRecord]:
        """Records of ``count`` consecutive chunks starting at ``tokens[first_start]``."""
        width = self.chunk_size
        rows = np.asarray(tokens[first_start : first_start + count * width], dtype=np.int64)
        if rows.shape[0] != count * width:
            raise ValueError(f"fingerprint requires {count * width} tokens, got {rows.shape[0]}")
        rows = rows.reshape(count, width)
        hashes = chunk_hashes(rows).tolist()
        return [
            FingerprintRecord(SegmentId(model_scope, hashes[i], first_start + i * width, width),
                              tuple(rows[i].tolist()))
            for i in range(count)
        ]

    def register(self, record: FingerprintRecord) -> None:
        with self._lock:
            current = self._records.get(record.segment_id)
            if current == record:
                return
            if current is not None:
                self.unregister(record.segment_id)
            sid = record.segment_id
            self._records[sid] = record
            self._by_hash[(sid.model_scope, sid.content_hash)].append(record)
            self._hashes[sid.model_scope].add(sid.content_hash)

    def unregister(self, segment_id: SegmentId) -> None:
        with self._lock:
            if self._records.pop(segment_id, None) is None:
                return
            key = (segment_id.model_scope, segment_id.content_hash)
            remaining = [r for r in self._by_hash[key] if r.segment_id != segment_id]
            if remaining:
                self._by_hash[key] = remaining
                return
            del self._by_hash[key]
            scope = self._hashes[segment_id.model_scope]
            scope.discard(segment_id.content_hash)
            if not scope:
                del self._hashes[segment_id.model_scope]

    def match(
        self, model_scope: str, tokens: Sequence[int], start_offset: int = 0
    ) -> tuple[BlendSegment, ...]:
        if not 0 <= start_offset <= len(tokens):
            raise ValueError("start_offset is outside the token sequence")
        found: list[BlendSegment] = []
        with self._lock:
            known = self._hashes.get(model_scope)
            if not known:
                return ()
            hashes = window_hashes(np.asarray(tokens[start_offset:], dtype=np.int64), self.chunk_size)
            wanted = np.fromiter(known, dtype=np.uint64, count=len(known))
            next_free = start_offset
            for rel in np.flatnonzero(np.isin(hashes, wanted)):
                target = start_offset + int(rel)
                if target < next_free:
                    continue
                candidates = self._by_hash.get((model_scope, int(hashes[rel])), ())
                window = tuple(int(t) for t in tokens[target : target + self.chunk_size])
                record = next((r for r in candidates if r.tokens == window), None)
                if record is None:
                    continue
                found.append(BlendSegment(record.segment_id, target))
                next_free = target + self.chunk_size
        return tuple(found)

    def validate(self, segments: Iterable[BlendSegment]) -> tuple[BlendSegment, ...]:
        with self._lock:
            return tuple(seg for seg in segments if seg.segment_id in self._records)

    def __len__(self) -> int:
        with self._lock:
            return len(self._records)
