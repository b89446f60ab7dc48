"""Token scoring and recompute selection (K3; K4 host side).

* ``kv_deviation`` -- ``cb_kv_deviation``: fp32 sum over the flattened local
  heads of (k_fresh - k_cached)^2 per active token (ascend.py:535-538).
* ``recompute_budget`` -- the top-k budget of ``_select`` (ascend.py:775-786):
  ``k = int(cached * ratio)`` clamped to ``[1, available]`` when both counts
  are non-zero, else 0; forced tokens do not consume budget.
* ``select_tokens`` -- optional TP all-reduce of the scores (every rank then
  runs the same deterministic kernel, so the reference's rank-0 broadcast is
  unnecessary) and ``cb_select_topk``: ascending indices of base ∪ top-k.
  With a ``PeerScoreExchange`` the all-reduce runs inside the select kernel
  over NVLink peer memory (``cb_select_topk_peer``).
* ``deviation_select`` -- both in one launch (``cb_kv_deviation_select``) when
  no all-reduce sits between them (one rank, or per-rank selection).
* ``sparse_q_masks`` -- query set, forced set and tail fallback of
  ``_sparse_q_scores`` (ascend.py:652-673); these depend only on the plan's
  gap mask, so they are computed on the host without a device round trip.

Host arrays reach the device through pinned staging (``_upload``): a copy from
pageable memory would wait for the stream, i.e. synchronise the host with the
GPU in the middle of the scoring path.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native


def _upload(array: np.ndarray, device) -> torch.Tensor:
    """Host array -> device tensor, asynchronously through pinned memory (torch's
    pinned-memory cache keeps the staging alive until the copy has run)."""
    return torch.from_numpy(np.ascontiguousarray(array)).pin_memory().to(device, non_blocking=True)


def _as_host_mask(mask: torch.Tensor | np.ndarray, name: str) -> np.ndarray:
    if isinstance(mask, np.ndarray):
        return mask.astype(np.bool_, copy=False)
    if mask.dtype != torch.bool:
        raise ValueError(f"{name} must be a boolean mask")
    return mask.detach().to("cpu").numpy()


def kv_deviation(
    fresh_key: torch.Tensor,
    cached_key: torch.Tensor,
    absolute_indices: torch.Tensor | None = None,
    absolute_offset: int = 0,
    out: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> torch.Tensor:
    """fp32 K-deviation score per row of ``fresh_key`` ([T, W] vs cached [N, W])."""
    _native.require_cuda(fresh_key, cached_key)
    fresh = fresh_key.reshape(fresh_key.shape[0], -1)
    cached = cached_key.reshape(cached_key.shape[0], -1)
    if fresh.shape[1] != cached.shape[1]:
        raise ValueError("fresh and cached keys must have the same row width")
    if fresh.dtype != cached.dtype:
        raise ValueError("fresh and cached keys must have the same dtype")
    if fresh.stride(1) != 1:
        fresh = fresh.contiguous()
    if cached.stride(1) != 1:
        cached = cached.contiguous()
    tokens = fresh.shape[0]
    if out is None:
        out = torch.empty(tokens, dtype=torch.float32, device=fresh.device)
    index_ptr = 0
    if absolute_indices is not None:
        absolute_indices = absolute_indices.to(device=fresh.device, dtype=torch.long).contiguous()
        if absolute_indices.numel() != tokens:
            raise ValueError("one absolute index per fresh key row is required")
        index_ptr = absolute_indices.data_ptr()
    esize = fresh.element_size()
    _native.call(
        "cb_kv_deviation",
        fresh.data_ptr(),
        fresh.stride(0) * esize,
        cached.data_ptr(),
        cached.stride(0) * esize,
        cached.shape[0],
        index_ptr,
        absolute_offset,
        tokens,
        fresh.shape[1],
        _native.dtype_code(fresh.dtype),
        out.data_ptr(),
        _native.stream_handle(stream),
    )
    return out


def recompute_budget(active: int, gap_count: int, base_count: int, ratio: float) -> int:
    """Top-k size of ``_select`` (forced tokens are free, gaps never count)."""
    cached = active - gap_count
    available = active - base_count
    if not cached or not available:
        return 0
    return min(max(int(cached * ratio), 1), available)


def select_from_scores(
    scores: torch.Tensor,
    base_mask: torch.Tensor,
    k: int,
    selected_count: int,
    stream: torch.cuda.Stream | None = None,
) -> torch.Tensor:
    """``cb_select_topk``: int64 ascending indices of base ∪ top-k (device)."""
    _native.require_cuda(scores, base_mask)
    if scores.dtype != torch.float32 or not scores.is_contiguous():
        raise ValueError("scores must be a contiguous float32 vector")
    if base_mask.dtype != torch.uint8 or base_mask.numel() != scores.numel():
        raise ValueError("base mask must be a uint8 vector shaped like the scores")
    out = torch.empty(selected_count, dtype=torch.long, device=scores.device)
    if scores.numel() == 0:
        return out
    _native.call(
        "cb_select_topk",
        scores.data_ptr(),
        base_mask.data_ptr(),
        scores.numel(),
        k,
        out.data_ptr(),
        out.numel(),
        _native.stream_handle(stream),
    )
    return out


_FUSED_WORKSPACES: dict[torch.device, torch.Tensor] = {}


def _fused_workspace(device: torch.device) -> torch.Tensor:
    """The per-device workspace of cb_kv_deviation_select (zeroed once; every call
    leaves it zero again).  Calls on one device are stream-ordered by the caller."""
    workspace = _FUSED_WORKSPACES.get(device)
    if workspace is None:
        size = ctypes.c_int64(0)
        _native.call("cb_kv_deviation_select_workspace_size", ctypes.addressof(size))
        workspace = torch.zeros(size.value, dtype=torch.uint8, device=device)
        _FUSED_WORKSPACES[device] = workspace
    return workspace


def deviation_select(
    fresh_key: torch.Tensor,
    cached_key: torch.Tensor,
    gap_mask: torch.Tensor | np.ndarray,
    ratio: float,
    absolute_indices: torch.Tensor | None = None,
    absolute_offset: int = 0,
    stream: torch.cuda.Stream | None = None,
    base_mask_device: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """K-deviation scores and ``_select`` of one rank in a single launch
    (cb_kv_deviation_select): (ascending int64 indices, fp32 scores).  The budget
    comes from the host gap mask (ascend.py:775-786), so nothing is read back.
    ``base_mask_device``: the gap mask already on the device as uint8 (no upload;
    what a CUDA-graph capture needs)."""
    _native.require_cuda(fresh_key, cached_key)
    fresh = fresh_key.reshape(fresh_key.shape[0], -1)
    cached = cached_key.reshape(cached_key.shape[0], -1)
    if fresh.shape[1] != cached.shape[1]:
        raise ValueError("fresh and cached keys must have the same row width")
    if fresh.dtype != cached.dtype:
        raise ValueError("fresh and cached keys must have the same dtype")
    if fresh.stride(1) != 1:
        fresh = fresh.contiguous()
    if cached.stride(1) != 1:
        cached = cached.contiguous()
    gaps = _as_host_mask(gap_mask, "gap_mask")
    tokens = fresh.shape[0]
    if gaps.shape[0] != tokens:
        raise ValueError("gap mask must match the fresh key rows")
    gap_count = int(gaps.sum())
    k = recompute_budget(tokens, gap_count, gap_count, ratio)
    device = fresh.device
    scores = torch.empty(tokens, dtype=torch.float32, device=device)
    selected = torch.empty(gap_count + k, dtype=torch.long, device=device)
    if tokens == 0:
        return selected, scores
    index_ptr = 0
    if absolute_indices is not None:
        absolute_indices = absolute_indices.to(device=device, dtype=torch.long).contiguous()
        if absolute_indices.numel() != tokens:
            raise ValueError("one absolute index per fresh key row is required")
        index_ptr = absolute_indices.data_ptr()
    if base_mask_device is None:
        base = _upload(gaps.astype(np.uint8), device)
    else:
        if base_mask_device.dtype != torch.uint8 or base_mask_device.numel() != tokens:
            raise ValueError("base mask must be a uint8 vector shaped like the fresh rows")
        base = base_mask_device
    workspace = _fused_workspace(device)
    esize = fresh.element_size()
    _native.call(
        "cb_kv_deviation_select", fresh.data_ptr(), fresh.stride(0) * esize, cached.data_ptr(),
        cached.stride(0) * esize, cached.shape[0], index_ptr, absolute_offset, tokens, fresh.shape[1],
        _native.dtype_code(fresh.dtype), base.data_ptr(), k, scores.data_ptr(), selected.data_ptr(),
        selected.numel(), workspace.data_ptr(), workspace.numel(), _native.stream_handle(stream),
    )
    return selected, scores


def tp_all_reduce(scores: torch.Tensor, tp_group) -> torch.Tensor:
    """Sum partial per-token scores over the TP ranks (NCCL over NVLink)."""
    if hasattr(tp_group, "all_reduce") and hasattr(tp_group, "world_size"):
        return tp_group.all_reduce(scores)  # vLLM GroupCoordinator
    import torch.distributed as dist

    dist.all_reduce(scores, group=tp_group)
    return scores


def tp_world_size(tp_group) -> int:
    if tp_group is None:
        return 1
    if hasattr(tp_group, "world_size"):
        return int(tp_group.world_size)
    import torch.distributed as dist

    return dist.get_world_size(tp_group)


def select_tokens(
    scores: torch.Tensor,
    gap_mask: torch.Tensor | np.ndarray,
    ratio: float,
    forced_mask: torch.Tensor | np.ndarray | None = None,
    tp_group=None,
    global_selection: bool = True,
    base_mask_device: torch.Tensor | None = None,
    peer_exchange=None,
) -> torch.Tensor:
    """Full ``_select``: TP reduction, budget, masked top-k, ascending union.

    With a ``peer_exchange`` (``PeerScoreExchange`` of the TP group) the
    reduction runs inside the select kernel over NVLink peer memory instead of
    a NCCL all-reduce; ``scores`` are then this rank's partial scores."""
    use_peer = peer_exchange is not None and global_selection
    if global_selection and tp_world_size(tp_group) > 1 and not use_peer:
        scores = tp_all_reduce(scores, tp_group)
    gaps = _as_host_mask(gap_mask, "gap_mask")
    base = gaps.copy()
    if forced_mask is not None:
        forced = _as_host_mask(forced_mask, "forced_mask")
        if forced.shape != gaps.shape:
            raise ValueError("forced selection mask must match the active token shape")
        base |= forced
    active = scores.numel()
    if gaps.shape[0] != active:
        raise ValueError("gap mask must match the score vector")
    base_count = int(base.sum())
    k = recompute_budget(active, int(gaps.sum()), base_count, ratio)
    if base_mask_device is None:
        base_mask_device = _upload(base.astype(np.uint8), scores.device)
    if use_peer:
        return peer_exchange.select(scores.contiguous(), base_mask_device, k, base_count + k)
    return select_from_scores(scores.contiguous(), base_mask_device, k, base_count + k)


def sparse_q_masks(
    gap_mask: np.ndarray, block_size: int, overflow_blocks: int, tail_query_tokens: int
) -> tuple[np.ndarray, np.ndarray, bool]:
    """(query mask, forced mask, tail_fallback) of the Sparse-Q selector.

    Queries are the gap tokens; without gaps the last ``tail_query_tokens``
    tokens act as queries and are forced.  With gaps, every token within
    ``overflow_blocks * block_size`` of a gap is forced too.
    """
    gaps = gap_mask.astype(np.bool_, copy=False)
    query = gaps.copy()
    forced = gaps.copy()
    has_gap = bool(gaps.any())
    if not has_gap:
        # same slice as ascend.py:659-660, including x[-0:] meaning "all"
        tail = min(tail_query_tokens, gaps.shape[0])
        query[-tail:] = True
        forced[-tail:] = True
    radius = overflow_blocks * block_size
    if radius and has_gap:
        counts = np.concatenate(([0], np.cumsum(gaps, dtype=np.int64)))
        index = np.arange(gaps.shape[0])
        left = np.clip(index - radius, 0, None)
        right = np.clip(index + radius + 1, None, gaps.shape[0])
        forced |= counts[right] > counts[left]
    return query, forced, not has_gap


def sparse_q_workspace_bytes(num_queries: int, num_q_heads: int, num_kv_heads: int,
                             head_size: int, dtype: torch.dtype) -> int:
    out = ctypes.c_int64(0)
    _native.call(
        "cb_sparse_q_workspace_size", num_queries, num_q_heads, num_kv_heads, head_size,
        _native.dtype_code(dtype), ctypes.addressof(out),
    )
    return int(out.value)


def sparse_q_key_mass(
    query: torch.Tensor,
    key: torch.Tensor,
    query_rows: np.ndarray,
    query_positions: np.ndarray,
    scale: float,
    workspace: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> torch.Tensor:
    """fp32 [num_keys] attention mass per key from the given sparse queries (cb_sparse_q_scores)."""
    _native.require_cuda(query, key)
    if query.ndim != 3 or key.ndim != 3:
        raise ValueError("query must be [tokens, q_heads, head] and key [keys, kv_heads, head]")
    if query.dtype != key.dtype:
        raise ValueError("query and key must share a dtype (one tcgen05 operand type)")
    if query.stride(-1) != 1 or query.stride(-2) != query.shape[-1]:
        raise ValueError("query heads must be contiguous")
    if key.stride(-1) != 1 or key.stride(-2) != key.shape[-1]:
        raise ValueError("key heads must be contiguous")
    rows = np.ascontiguousarray(query_rows, dtype=np.int64)
    positions = np.ascontiguousarray(query_positions, dtype=np.int64)
    num_keys = key.shape[0]
    if rows.shape != positions.shape:
        raise ValueError("one position per query row is required")
    if rows.size and (rows.min() < 0 or rows.max() >= query.shape[0]):
        raise IndexError("query row out of range")
    if positions.size and (positions.min() < 0 or positions.max() >= num_keys):
        raise IndexError("query position outside the key context")
    num_q_heads, head = query.shape[1], query.shape[2]
    num_kv_heads = key.shape[1]
    needed = sparse_q_workspace_bytes(rows.size, num_q_heads, num_kv_heads, head, query.dtype)
    if workspace is None or workspace.numel() < needed:
        workspace = torch.empty(needed + 1024, dtype=torch.uint8, device=query.device)
    base = workspace.data_ptr()
    aligned = (base + 1023) // 1024 * 1024
    usable = workspace.numel() - (aligned - base)
    scores = torch.empty(num_keys, dtype=torch.float32, device=query.device)
    rows_dev = _upload(rows, query.device)
    pos_dev = _upload(positions, query.device)
    esize = query.element_size()
    _native.call(
        "cb_sparse_q_scores",
        query.data_ptr(), query.stride(0) * esize, query.shape[0], key.data_ptr(), key.stride(0) * esize,
        num_keys,
        num_q_heads, num_kv_heads, head, _native.dtype_code(query.dtype), rows_dev.data_ptr(),
        pos_dev.data_ptr(), rows.size, float(scale), scores.data_ptr(), aligned, usable,
        0 if device_error is None else device_error.data_ptr(), _native.stream_handle(stream),
    )
    return scores


def sparse_q_scores(
    query: torch.Tensor,
    key: torch.Tensor,
    absolute_indices: torch.Tensor | np.ndarray,
    gap_mask: torch.Tensor | np.ndarray,
    scale: float,
    block_size: int,
    overflow_blocks: int,
    tail_query_tokens: int,
    device_error: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, dict[str, int | bool]]:
    """``_sparse_q_scores`` (ascend.py:638-711): scores of the active tokens (device
    fp32), forced mask (host bool tensor), stats.

    ``absolute_indices`` and ``gap_mask`` are best given as host arrays (the
    executor keeps them there): the query rows, forced mask and budgets then
    come from host data, and the scoring enqueues without any device read.
    ``query_score_chunk_size`` only bounded the reference's temporary tensor;
    the tensor-core kernel streams keys through TMEM and never materialises a
    [queries, context] tensor, so it has no chunk parameter.
    """
    gaps = _as_host_mask(gap_mask, "gap_mask")
    absolute = (
        np.asarray(absolute_indices, dtype=np.int64)
        if isinstance(absolute_indices, np.ndarray)
        else absolute_indices.detach().to("cpu", torch.long).numpy()
    )
    if gaps.shape[0] != query.shape[0] or absolute.shape[0] != query.shape[0]:
        raise ValueError("gap mask and absolute indices must match the active tokens")
    query_mask, forced, tail_fallback = sparse_q_masks(
        gaps, block_size, overflow_blocks, tail_query_tokens
    )
    rows = np.flatnonzero(query_mask)
    full = sparse_q_key_mass(query, key, rows, absolute[rows], scale, device_error=device_error)
    count = absolute.shape[0]
    if count and np.array_equal(absolute, np.arange(absolute[0], absolute[0] + count)):
        scores = full[int(absolute[0]) : int(absolute[0]) + count]  # the span: a view, no gather
    else:
        scores = full.index_select(0, _upload(absolute, query.device))
    gap_count = int(gaps.sum())
    stats = {
        "active_tokens": int(query.shape[0]),
        "gap_tokens": gap_count,
        "cached_tokens": int(query.shape[0]) - gap_count,
        "sparse_query_tokens": int(rows.size),
        "tail_fallback": tail_fallback,
        "overflow_blocks": overflow_blocks,
    }
    return scores, torch.from_numpy(forced), stats


def selection_overlap(a: torch.Tensor, b: torch.Tensor) -> tuple[int, int]:
    """(overlap, union) of two ascending selections on the device (cb_sorted_overlap):
    the ``compare`` strategy's diagnostic (ascend.py:713-747) with one 8-byte read back
    instead of two boolean masks and three synchronisations."""
    _native.require_cuda(a, b)
    a = a.to(torch.long).contiguous()
    b = b.to(device=a.device, dtype=torch.long).contiguous()
    count = torch.empty(1, dtype=torch.long, device=a.device)
    _native.call("cb_sorted_overlap", a.data_ptr(), a.numel(), b.data_ptr(), b.numel(), count.data_ptr(),
                 _native.stream_handle())
    overlap = int(count.item())
    return overlap, a.numel() + b.numel() - overlap
