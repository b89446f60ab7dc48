"""CPU oracle of the CacheBlend hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline / reference
legs of bench.py may import this package, and only as the checker or the
timed CPU baseline.  The product (pic-kvcache_b200/cacheblend_b200) never
imports, links or calls it.

It restates the reference (zoudinghong2000/PIC-KVCache, ``cacheblend_vllm``)
on numpy arrays:

* byte/bf16 work in plain C (``cb_oracle.c``, built by ``build()`` with gcc,
  OpenMP over tokens): paged gather/scatter (kv_layout.py:90-161), RoPE
  relocation (ascend.py:52-103), the per-layer blend load
  (ascend.py:224-287, 313-370) and the K-deviation score (ascend.py:535-538);
* selection in numpy: the ``_select`` budget and masked top-k
  (ascend.py:757-796), ties resolved towards the lowest index;
* Sparse-Q scoring in numpy (ascend.py:638-711): bf16-rounded Q.K^T logits,
  fp32 scale, causal mask, fp32 softmax, mass summed per key.

Pinned against the reference: tests/golden/ holds vectors produced by the
reference itself (tests/golden/make_golden.py) and the reference's own
known-answer tests; tests/test_oracle_golden.py checks this oracle against
them.  bf16 values are carried as uint16 bit patterns.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "cb_oracle.c"
LIB_PATH = ORACLE_DIR / "_build" / "libcb_oracle.so"

BF16, FP16, FP32 = 0, 1, 2
_NP_STORAGE = {BF16: np.uint16, FP16: np.float16, FP32: np.float32}

_lib: ctypes.CDLL | None = None
_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int


def build(force: bool = False) -> Path:
    """Compile cb_oracle.c with gcc (-O3 -fopenmp -ffp-contract=off)."""
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB_PATH
    LIB_PATH.parent.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    compilers = [c for c in ("/usr/bin/gcc", os.environ.get("CC"), "gcc") if c]
    errors = []
    # OpenMP first; a compiler without libgomp still yields a (serial) oracle
    for openmp in (True, False):
        for compiler in compilers:
            cmd = [compiler, "-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
                   str(SOURCE), "-o", str(tmp), "-lm"]
            if openmp:
                cmd.insert(1, "-fopenmp")
            proc = subprocess.run(cmd, capture_output=True, text=True)
            if proc.returncode == 0:
                os.replace(tmp, LIB_PATH)
                return LIB_PATH
            errors.append(f"{' '.join(cmd)}: {proc.stderr.strip()[:200]}")
    raise RuntimeError("could not compile the oracle:\n" + "\n".join(errors))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        handle = ctypes.CDLL(str(build()))
        handle.orc_threads.restype = _i32
        handle.orc_threads.argtypes = [_i32]
        handle.orc_paged_gather.restype = _i32
        handle.orc_paged_gather.argtypes = [_p, _p] + [_i64] * 7 + [_p, _i64, _p] + [_i64] * 3 + [_i32]
        handle.orc_paged_scatter.restype = _i32
        handle.orc_paged_scatter.argtypes = [_p] + [_i64] * 3 + [_p, _p] + [_i64] * 7 + [_p, _i64]
        handle.orc_relocate.restype = _i32
        handle.orc_relocate.argtypes = [_i32, _p, _p] + [_i64] * 4 + [_i32, _p, _i64, _p, _p, _i32]
        handle.orc_blend_load.restype = _i32
        handle.orc_blend_load.argtypes = (
            [_i32, _p, _i64, _i64, _p, _p] + [_i64] * 5 + [_p] + [_i64] * 3
            + [_i32, _p, _i64, _i64] + [_p] * 6 + [_i32]
        )
        handle.orc_kv_deviation.restype = _i32
        handle.orc_kv_deviation.argtypes = [_i32, _p, _i64, _p, _i64, _p] + [_i64] * 4 + [_p, _i32]
        _lib = handle
    return _lib


def threads(requested: int = 0) -> int:
    return int(lib().orc_threads(requested))


def _ptr(array: np.ndarray) -> int:
    return array.ctypes.data


# ---------------------------------------------------------------- bf16 helpers
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (quiet NaN preserved)."""
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    quiet = ((u >> 16) | 0x40).astype(np.uint16)
    return np.where(nan, quiet, rounded)


def round_bf16(values: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(values))


def to_f32(array: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == BF16:
        return bf16_to_f32(array)
    return array.astype(np.float32)


# ---------------------------------------------------------------- paged copies
def _plane_geometry(key: np.ndarray) -> tuple[int, int, int, int, int]:
    """(block_stride, slot_stride, heads, head_bytes, head_stride) of [NB, BS, *row]."""
    esize = key.itemsize
    row = key.shape[2:]
    if len(row) == 0:
        return key.strides[0], key.strides[1], 1, esize, esize
    if len(row) == 1:
        return key.strides[0], key.strides[1], 1, row[0] * esize, row[0] * esize
    if key.strides[-1] != esize:
        raise ValueError("oracle needs a contiguous innermost dim")
    heads = int(np.prod(row[:-1]))
    return key.strides[0], key.strides[1], heads, row[-1] * esize, key.strides[-2]


def paged_gather(key: np.ndarray, value: np.ndarray, slots: np.ndarray, block_size: int,
                 nthreads: int = 0) -> np.ndarray:
    """out[p, t] = plane_p[slot // block_size, slot % block_size]."""
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    bstride, sstride, heads, head_bytes, hstride = _plane_geometry(key)
    out = np.empty((2, slots.shape[0], *key.shape[2:]), dtype=key.dtype)
    row_bytes = heads * head_bytes
    rc = lib().orc_paged_gather(
        _ptr(key), _ptr(value), bstride, sstride, hstride, key.shape[0], block_size, heads,
        head_bytes, _ptr(slots), slots.shape[0], _ptr(out), slots.shape[0] * row_bytes, row_bytes,
        head_bytes, nthreads,
    )
    if rc:
        raise IndexError("slot out of range")
    return out


def paged_scatter(contiguous: np.ndarray, key: np.ndarray, value: np.ndarray, slots: np.ndarray,
                  block_size: int) -> None:
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    contiguous = np.ascontiguousarray(contiguous)
    bstride, sstride, heads, head_bytes, hstride = _plane_geometry(key)
    row_bytes = heads * head_bytes
    rc = lib().orc_paged_scatter(
        _ptr(contiguous), slots.shape[0] * row_bytes, row_bytes, head_bytes, _ptr(key),
        _ptr(value), bstride, sstride, hstride, key.shape[0], block_size, heads, head_bytes,
        _ptr(slots), slots.shape[0],
    )
    if rc:
        raise IndexError("slot out of range")


# ---------------------------------------------------------------- relocation
def relocate(key: np.ndarray, cos_sin: np.ndarray, old: np.ndarray, new: np.ndarray,
             head_size: int, rotary_dim: int, neox: bool, dtype: int,
             nthreads: int = 0) -> np.ndarray:
    """R(new) R(old)^-1 key, op by op in ``dtype``; key [T, heads*head_size]."""
    key = np.ascontiguousarray(key)
    cos_sin = np.ascontiguousarray(cos_sin)
    old = np.ascontiguousarray(old, dtype=np.int64)
    new = np.ascontiguousarray(new, dtype=np.int64)
    out = np.empty_like(key)
    tokens = key.shape[0]
    heads = key.size // max(tokens, 1) // head_size if tokens else 1
    rc = lib().orc_relocate(
        dtype, _ptr(key), _ptr(out), tokens, heads, head_size, rotary_dim, int(neox),
        _ptr(cos_sin), cos_sin.shape[0], _ptr(old), _ptr(new), nthreads,
    )
    if rc:
        raise IndexError("position outside the RoPE cos_sin_cache")
    return out


def blend_load(dtype: int, alloc_end: int, apc_prefix: int, key_cache: np.ndarray,
               value_cache: np.ndarray, slots: np.ndarray, block_size: int,
               segments: list[tuple[int, int, int, np.ndarray]], rotate: np.ndarray,
               cos_sin: np.ndarray, head_size: int, rotary_dim: int, neox: bool,
               nthreads: int = 0) -> np.ndarray:
    """Staging [2, alloc_end, *row] of one layer.

    ``segments``: (source_start, target_start, length, host chunk [2, length, *row]).
    """
    row = key_cache.shape[2:]
    out = np.empty((2, alloc_end, *row), dtype=key_cache.dtype)
    width = int(np.prod(row))
    heads = width // head_size
    bstride, sstride, _, _, hstride = _plane_geometry(key_cache)
    hosts = [np.ascontiguousarray(seg[3]) for seg in segments]
    src = np.array([s[0] for s in segments], dtype=np.int64)
    tgt = np.array([s[1] for s in segments], dtype=np.int64)
    length = np.array([s[2] for s in segments], dtype=np.int64)
    k_src = np.array([h[0].ctypes.data for h in hosts], dtype=np.uint64)
    v_src = np.array([h[1].ctypes.data for h in hosts], dtype=np.uint64)
    rot = np.ascontiguousarray(rotate, dtype=np.int32)
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    cos_sin = np.ascontiguousarray(cos_sin)
    rc = lib().orc_blend_load(
        dtype, _ptr(out), alloc_end, apc_prefix, _ptr(key_cache), _ptr(value_cache), bstride,
        sstride, hstride, key_cache.shape[0], block_size, _ptr(slots), heads, head_size,
        rotary_dim, int(neox), _ptr(cos_sin), cos_sin.shape[0], len(segments), _ptr(src),
        _ptr(tgt), _ptr(length), _ptr(rot), _ptr(k_src), _ptr(v_src), nthreads,
    )
    if rc:
        raise IndexError("blend plan outside the staging or RoPE table")
    return out


# ---------------------------------------------------------------- scoring
def kv_deviation(fresh: np.ndarray, cached: np.ndarray, dtype: int,
                 abs_index: np.ndarray | None = None, abs_offset: int = 0,
                 unit: int | None = None, nthreads: int = 0) -> np.ndarray:
    """fp32 sum of squared differences per fresh row (kernel association order)."""
    fresh = np.ascontiguousarray(fresh).reshape(fresh.shape[0], -1)
    cached = np.ascontiguousarray(cached).reshape(cached.shape[0], -1)
    width = fresh.shape[1]
    if unit is None:
        unit = 16 // fresh.itemsize if (width * fresh.itemsize) % 16 == 0 else 1
    idx = None if abs_index is None else np.ascontiguousarray(abs_index, dtype=np.int64)
    out = np.empty(fresh.shape[0], dtype=np.float32)
    rc = lib().orc_kv_deviation(
        dtype, _ptr(fresh), fresh.strides[0], _ptr(cached), cached.strides[0],
        None if idx is None else _ptr(idx), abs_offset, fresh.shape[0], width, unit, _ptr(out),
        nthreads,
    )
    if rc:
        raise ValueError("width is not a multiple of the unit")
    return out


def recompute_budget(active: int, gap_count: int, base_count: int, ratio: float) -> int:
    """``_select`` budget (ascend.py:775-786)."""
    cached = active - gap_count
    available = active - base_count
    k = int(cached * ratio)
    if cached and available:
        return min(max(k, 1), available)
    return 0


def select(scores: np.ndarray, gap_mask: np.ndarray, ratio: float,
           forced_mask: np.ndarray | None = None) -> np.ndarray:
    """Ascending indices of gaps ∪ forced ∪ top-k cached scores (ties: lowest index)."""
    scores = np.asarray(scores, dtype=np.float32)
    base = np.asarray(gap_mask, dtype=np.bool_).copy()
    if forced_mask is not None:
        base |= np.asarray(forced_mask, dtype=np.bool_)
    k = recompute_budget(scores.shape[0], int(np.sum(gap_mask)), int(base.sum()), ratio)
    chosen = base.copy()
    if k:
        candidates = np.flatnonzero(~base)
        values = scores[candidates].astype(np.float64)
        nan = np.isnan(values)  # NaN ranks above +inf (torch.topk order)
        values = np.where(nan, 0.0, values) + 0.0  # -0.0 ties with +0.0
        order = np.lexsort((candidates, -values, ~nan))  # NaN, then descending, then index
        chosen[candidates[order[:k]]] = True
    return np.flatnonzero(chosen).astype(np.int64)


def sparse_q_masks(gap_mask: np.ndarray, block_size: int, overflow_blocks: int,
                   tail_query_tokens: int) -> tuple[np.ndarray, np.ndarray, bool]:
    """(query mask, forced mask, tail_fallback) of ascend.py:652-671."""
    gaps = np.asarray(gap_mask, dtype=np.bool_)
    query = gaps.copy()
    forced = gaps.copy()
    has_gap = bool(gaps.any())
    if not has_gap:
        tail = min(tail_query_tokens, gaps.shape[0])
        query[-tail:] = True
        forced[-tail:] = True
    radius = overflow_blocks * block_size
    if radius and has_gap:
        n = gaps.shape[0]
        for i in np.flatnonzero(gaps):
            forced[max(0, i - radius): min(n, i + radius + 1)] = True
    return query, forced, not has_gap


def sparse_q_key_mass(query: np.ndarray, key: np.ndarray, positions: np.ndarray, scale: float,
                      chunk: int = 8, dtype: int = BF16) -> np.ndarray:
    """Attention mass per key from the given queries (the loop of ascend.py:681-697), float64.

    query [Q, Hq, D] (the sparse queries, in order) and key [N, Hkv, D] as fp32
    arrays holding values of ``dtype``; positions [Q].  Per chunk of ``chunk`` queries
    and per (KV head, group): logits = T(q . k) * fp32 scale (T = the matmul output
    type, bf16 or fp16), keys after a query's
    position masked (their exp is exactly 0, as exp(finfo.min - max) is in the
    reference), fp32 softmax over the keys, summed per key.
    """
    q = np.asarray(query, dtype=np.float32)
    pos = np.asarray(positions, dtype=np.int64)
    heads, kv_heads = q.shape[1], key.shape[1]
    if heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    groups = heads // kv_heads
    keys = np.asarray(key, dtype=np.float32)
    total = np.zeros(key.shape[0], dtype=np.float64)
    scale32 = np.float32(scale)
    for start in range(0, q.shape[0], chunk):
        stop = min(start + chunk, q.shape[0])
        limit = int(pos[start:stop].max()) + 1
        masked = pos[start:stop, None] < np.arange(limit)[None, :]
        block = np.zeros(limit, dtype=np.float64)
        for h in range(kv_heads):
            k_h = keys[:limit, h, :]  # [limit, D]
            for g in range(groups):
                logits = _round_to(q[start:stop, h * groups + g, :] @ k_h.T, dtype) * scale32
                logits[masked] = -np.inf
                e = np.exp(logits - logits.max(axis=1, keepdims=True), dtype=np.float32)
                probs = e / e.sum(axis=1, keepdims=True, dtype=np.float32)
                block += probs.sum(axis=0, dtype=np.float64)
        total[:limit] += block
    return total


def sparse_q_scores(query: np.ndarray, key: np.ndarray, absolute: np.ndarray,
                    gap_mask: np.ndarray, scale: float, block_size: int, overflow_blocks: int,
                    tail_query_tokens: int, chunk: int = 8,
                    full: bool = False) -> tuple[np.ndarray, np.ndarray, dict]:
    """Sparse-Q attention mass per key (ascend.py:638-711), numpy fp32.

    query [A, Hq, D] and key [N, Hkv, D] as fp32 arrays holding bf16 values.
    Queries are the gap tokens (or the tail, ascend.py:652-673); their mass per
    key comes from ``sparse_q_key_mass``.  Returns the per-active-token scores
    (or the full per-key vector when ``full``), the forced mask and the stats.
    """
    query_mask, forced, tail_fallback = sparse_q_masks(
        gap_mask, block_size, overflow_blocks, tail_query_tokens
    )
    rows = np.flatnonzero(query_mask)
    pos = np.asarray(absolute, dtype=np.int64)[rows]
    total = sparse_q_key_mass(query[rows], key, pos, scale, chunk)
    stats = {
        "active_tokens": int(query.shape[0]),
        "gap_tokens": int(np.sum(gap_mask)),
        "cached_tokens": int(query.shape[0] - np.sum(gap_mask)),
        "sparse_query_tokens": int(rows.shape[0]),
        "tail_fallback": tail_fallback,
        "overflow_blocks": overflow_blocks,
    }
    scores = total.astype(np.float32)
    if full:
        return scores, forced, stats
    return scores[np.asarray(absolute, dtype=np.int64)], forced, stats


def _round_to(values: np.ndarray, dtype: int) -> np.ndarray:
    """fp32 values rounded to the element type (nearest even), returned as fp32."""
    if dtype == BF16:
        return round_bf16(values)
    if dtype == FP16:
        return values.astype(np.float16).astype(np.float32)
    return values.astype(np.float32)


def blend_attention(query: np.ndarray, key: np.ndarray, value: np.ndarray, positions: np.ndarray,
                    scale: float, dtype: int = BF16) -> np.ndarray:
    """Attention of the computed queries over the staging context
    (Qwen3BlendExecutor._attention, ascend.py:798-846, einsum path), numpy fp32.

    query [Nq, Hq, D], key / value [Nk, Hkv, D] as fp32 arrays holding values
    of the element type; query head h uses KV head h // (Hq // Hkv).  Each
    step rounds where the reference's tensors do: the Q.K^T product to the
    element type, the scaled logits to the element type, softmax in fp32 over
    keys k <= position (masked logits contribute exp(finfo.min - max) == 0),
    probabilities to the element type, the P.V product to the element type.
    Returns fp32 values of the element type.
    """
    nq, hq, _ = query.shape
    nk, hkv, _ = key.shape
    if hq % hkv:
        raise ValueError("query heads must be divisible by KV heads")
    groups = hq // hkv
    pos = np.asarray(positions, dtype=np.int64)
    scale32 = np.float32(scale)
    out = np.zeros(query.shape, dtype=np.float32)
    for start in range(0, nq, 128):
        rows = slice(start, min(start + 128, nq))
        limit = int(pos[rows].max()) + 1
        masked = pos[rows, None] < np.arange(limit)[None, :]
        for h in range(hkv):
            k_h = key[:limit, h, :].astype(np.float32)
            v_h = value[:limit, h, :].astype(np.float32)
            for g in range(groups):
                q = query[rows, h * groups + g, :].astype(np.float32)
                logits = _round_to(_round_to(q @ k_h.T, dtype) * scale32, dtype)
                logits[masked] = -np.inf
                e = np.exp(logits - logits.max(axis=1, keepdims=True), dtype=np.float32)
                probs = _round_to(e / e.sum(axis=1, keepdims=True, dtype=np.float32), dtype)
                out[rows, h * groups + g, :] = probs @ v_h
    return _round_to(out, dtype)
