"""Content fingerprints and the token-range matcher behind the store.

The fingerprint function is part of the store's wire contract: segment ids
(and therefore cache hits across processes) depend on it.  It is the 64-bit
polynomial hash of cacheblend_vllm/hashing.py:18-22 -- base 1,000,003 over
``token + 1``, wrapping modulo 2**64.  Window hashes at every offset come from
one rolling pass in the native library (``cb_window_hashes``, O(N) instead of
the reference's O(N x window) sliding matmul, hashing.py:42-53), and the
offsets whose hash is committed from a binary-search scan over the sorted
committed hashes (``cb_hash_candidates``); both are host code, no GPU.

Matching semantics follow TokenRangeMatcher.match (matcher.py:80-125):
leftmost-greedy, non-overlapping, with exact token verification.
"""

from __future__ import annotations

import array
import functools
import threading
from collections import defaultdict
from collections.abc import Iterable, Sequence
from dataclasses import dataclass

import ctypes

import numpy as np

from . import _native
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


@functools.lru_cache(maxsize=16)
def _powers(base: int, count: int) -> np.ndarray:
    """[base**0, base**1, ..., base**(count-1)] modulo 2**64 as uint64 (read-only,
    cached: every chunk of one width shares the weights)."""
    out = np.empty(count, dtype=np.uint64)
    if count == 0:
        return out
    out[0] = 1
    if count > 1:
        out[1:] = np.uint64(base)
        with np.errstate(over="ignore"):
            np.cumprod(out, out=out)
    out.flags.writeable = False
    return out


def window_hashes(tokens: Sequence[int] | np.ndarray, window: int) -> np.ndarray:
    """uint64 fingerprint of every full window of ``tokens`` (O(N), native)."""
    if window <= 0:
        raise ValueError("window must be positive")
    values = np.ascontiguousarray(tokens, dtype=np.int64)
    n = values.shape[0]
    if n < window:
        return np.empty(0, dtype=np.uint64)
    out = np.empty(n - window + 1, dtype=np.uint64)
    _native.call("cb_window_hashes", values.ctypes.data, n, window, out.ctypes.data)
    return out


def hash_candidates(hashes: np.ndarray, known_sorted: np.ndarray) -> np.ndarray:
    """Ascending offsets whose hash is in ``known_sorted`` (ascending, distinct uint64)."""
    hashes = np.ascontiguousarray(hashes, dtype=np.uint64)
    known_sorted = np.ascontiguousarray(known_sorted, dtype=np.uint64)
    count = ctypes.c_int64(0)
    out = np.empty(min(hashes.shape[0], 4096), dtype=np.int64)
    while True:
        _native.call("cb_hash_candidates", hashes.ctypes.data, hashes.shape[0], known_sorted.ctypes.data,
                     known_sorted.shape[0], out.ctypes.data, out.shape[0], ctypes.addressof(count))
        if count.value <= out.shape[0]:
            return out[: count.value]
        out = np.empty(count.value, dtype=np.int64)


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
        self._sorted: dict[str, np.ndarray] = {}  # per scope: sorted committed hashes (lazy)
        self._token_rows: dict[SegmentId, np.ndarray] = {}  # per record: its tokens, for verification
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
        span = tokens[first_start : first_start + count * width]
        if isinstance(span, list):
            # a list of ints (vLLM's token ids): the record tuples are list slices
            rows = np.frombuffer(array.array("q", span), dtype=np.int64)
        else:
            rows = np.asarray(span, dtype=np.int64)
        if rows.shape[0] != count * width:
            raise ValueError(f"fingerprint requires {count * width} tokens, got {rows.shape[0]}")
        rows = rows.reshape(count, width)
        hashes = chunk_hashes(rows).tolist()
        if isinstance(span, list):
            chunks = [tuple(span[i * width : (i + 1) * width]) for i in range(count)]
        else:
            chunks = [tuple(row) for row in rows.tolist()]
        return [
            FingerprintRecord(SegmentId(model_scope, hashes[i], first_start + i * width, width), chunks[i])
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
            self._sorted.pop(sid.model_scope, None)
            self._token_rows[sid] = np.asarray(record.tokens, dtype=np.int64)

    def unregister(self, segment_id: SegmentId) -> None:
        with self._lock:
            if self._records.pop(segment_id, None) is None:
                return
            self._token_rows.pop(segment_id, None)
            key = (segment_id.model_scope, segment_id.content_hash)
            remaining = [r for r in self._by_hash[key] if r.segment_id != segment_id]
            if remaining:
                self._by_hash[key] = remaining
                return
            del self._by_hash[key]
            self._sorted.pop(segment_id.model_scope, None)
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
            wanted = self._sorted.get(model_scope)
            if wanted is None:
                wanted = np.sort(np.fromiter(known, dtype=np.uint64, count=len(known)))
                self._sorted[model_scope] = wanted
            values = np.asarray(tokens, dtype=np.int64)
            hashes = window_hashes(values[start_offset:], self.chunk_size)
            width = self.chunk_size
            next_free = start_offset
            for rel in hash_candidates(hashes, wanted).tolist():
                target = start_offset + rel
                if target < next_free:
                    continue
                window = values[target : target + width]
                record = next((r for r in self._by_hash.get((model_scope, int(hashes[rel])), ())
                               if np.array_equal(self._token_rows[r.segment_id], window)), None)
                if record is None:
                    continue
                found.append(BlendSegment(record.segment_id, target))
                next_free = target + width
        return tuple(found)

    def validate(self, segments: Iterable[BlendSegment]) -> tuple[BlendSegment, ...]:
        with self._lock:
            return tuple(seg for seg in segments if seg.segment_id in self._records)

    def __len__(self) -> int:
        with self._lock:
            return len(self._records)
