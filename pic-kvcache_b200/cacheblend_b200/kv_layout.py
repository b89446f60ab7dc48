"""Paged KV gather/scatter on B200 (K1).

Drop-in for cacheblend_vllm/kv_layout.py:90-161: ``gather_paged_kv`` and
``scatter_paged_kv`` take the same arguments, accept the same three vLLM
layouts -- merged-first ``[2, blocks, block_size, ...]`` (FlashAttention),
merged-block ``[blocks, 2, block_size, ...]`` (FlashInfer) and a separate
``(K, V)`` pair -- raise the same ``ValueError`` for anything else and return
``[2, tokens, ...]``.  The copy itself is one launch of ``cb_paged_gather`` /
``cb_paged_scatter`` over 16-byte vectors.  CUDA tensors only.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence
from dataclasses import dataclass

import torch

from . import _native

KVLayer = torch.Tensor | Sequence[torch.Tensor]


@dataclass(frozen=True)
class RowShape:
    """One token of one plane as ``num_heads`` rows of ``head_bytes`` bytes."""

    dims: tuple[int, ...]  # trailing tensor dims of a token, e.g. (H, D)
    num_heads: int
    head_bytes: int
    head_stride: int  # bytes
    element_size: int

    @property
    def row_bytes(self) -> int:
        return self.num_heads * self.head_bytes


@dataclass(frozen=True)
class PagedKV:
    """Byte-level description of one layer's paged K and V planes."""

    key: torch.Tensor  # [num_blocks, block_size_dim, *row]
    value: torch.Tensor
    block_stride: int
    slot_stride: int
    row: RowShape
    num_blocks: int
    block_dim: int
    block_size: int

    @property
    def dtype(self) -> torch.dtype:
        return self.key.dtype

    @property
    def device(self) -> torch.device:
        return self.key.device


def _row_shape(shape: Sequence[int], strides: Sequence[int], element_size: int) -> RowShape:
    """Express trailing dims as (heads, contiguous head bytes, head stride)."""
    dims = tuple(int(d) for d in shape)
    kept = [(int(d), int(st)) for d, st in zip(dims, strides) if d != 1]
    inner = 1  # elements of the contiguous innermost run
    while kept and kept[-1][1] == inner:
        inner *= kept.pop()[0]
    if not kept:
        return RowShape(dims, 1, inner * element_size, inner * element_size, element_size)
    heads, head_stride = kept[-1]
    for d, st in reversed(kept[:-1]):
        if st != head_stride * heads:
            raise ValueError(f"unsupported KV row strides {tuple(strides)} for shape {dims}")
        heads *= d
    return RowShape(dims, heads, inner * element_size, head_stride * element_size, element_size)


def match_rows(paged_row: RowShape, dense_row: RowShape) -> tuple[int, int, int, int]:
    """(num_heads, head_bytes, paged_head_stride, dense_head_stride) for one copy.

    A fully contiguous row can be split into any number of equal heads, so it
    adopts the other side's split; two strided rows must split the same way.
    """
    if paged_row.row_bytes != dense_row.row_bytes:
        raise ValueError("dense tensor row does not match the paged cache row")
    if dense_row.num_heads == 1:
        return paged_row.num_heads, paged_row.head_bytes, paged_row.head_stride, paged_row.head_bytes
    if paged_row.num_heads == 1:
        return dense_row.num_heads, dense_row.head_bytes, dense_row.head_bytes, dense_row.head_stride
    if (paged_row.num_heads, paged_row.head_bytes) != (dense_row.num_heads, dense_row.head_bytes):
        raise ValueError("dense tensor head layout does not match the paged cache")
    return paged_row.num_heads, paged_row.head_bytes, paged_row.head_stride, dense_row.head_stride


def _plane_pair(kv_layer: KVLayer) -> tuple[torch.Tensor, torch.Tensor]:
    """(K, V) views shaped [blocks, block_size, *row] for every supported layout."""
    if not isinstance(kv_layer, torch.Tensor):
        if len(kv_layer) != 2:
            raise ValueError(f"separate KV layout requires two tensors, got {len(kv_layer)}")
        key, value = kv_layer
        if not isinstance(key, torch.Tensor) or not isinstance(value, torch.Tensor):
            raise TypeError("separate KV layout must contain tensors")
        return key, value
    if kv_layer.shape[0] == 2:
        return kv_layer[0], kv_layer[1]
    if kv_layer.ndim >= 4 and kv_layer.shape[1] == 2:
        return kv_layer[:, 0], kv_layer[:, 1]
    raise ValueError(f"unsupported vLLM KV layout {tuple(kv_layer.shape)}")


def describe_paged(kv_layer: KVLayer, block_size: int) -> PagedKV:
    key, value = _plane_pair(kv_layer)
    if key.ndim < 2 or key.shape != value.shape or key.dtype != value.dtype:
        raise ValueError("K and V planes must have the same [blocks, block_size, ...] shape")
    if key.stride() != value.stride():
        raise ValueError("K and V planes must share strides")
    if key.device != value.device:
        raise ValueError("K and V planes must live on one device")
    if block_size <= 0 or block_size > key.shape[1]:
        raise ValueError(
            f"block_size {block_size} does not fit the cache block dimension {key.shape[1]}"
        )
    esize = key.element_size()
    row = _row_shape(key.shape[2:], key.stride()[2:], esize)
    return PagedKV(
        key=key,
        value=value,
        block_stride=key.stride(0) * esize,
        slot_stride=key.stride(1) * esize,
        row=row,
        num_blocks=int(key.shape[0]),
        block_dim=int(key.shape[1]),
        block_size=int(block_size),
    )


def device_slots(slot_mapping: torch.Tensor, paged: PagedKV, block_size: int) -> torch.Tensor:
    """int64 slots on the cache device; host-side slots are range-checked first."""
    num_slots = paged.num_blocks * block_size
    if slot_mapping.device.type == "cpu" and slot_mapping.numel():
        low = int(slot_mapping.min())
        high = int(slot_mapping.max())
        if low < -num_slots or high >= num_slots:
            raise IndexError(
                f"slot out of range for a paged cache of {num_slots} slots: [{low}, {high}]"
            )
    return slot_mapping.to(device=paged.device, dtype=torch.long, non_blocking=True).contiguous()


def dense_row(tensor: torch.Tensor) -> RowShape:
    return _row_shape(tensor.shape[2:], tensor.stride()[2:], tensor.element_size())


def gather_into(
    paged: PagedKV,
    slots: torch.Tensor,
    out: torch.Tensor,
    *,
    chunk_tokens: int = 0,
    chunk_stride: int = 0,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Launch cb_paged_gather into ``out`` ([2, T, *row]-strided, or chunk-major)."""
    heads, head_bytes, paged_hs, dense_hs = match_rows(paged.row, dense_row(out))
    esize = out.element_size()
    _native.call(
        "cb_paged_gather",
        paged.key.data_ptr(),
        paged.value.data_ptr(),
        paged.block_stride,
        paged.slot_stride,
        paged_hs,
        paged.num_blocks,
        paged.block_size,
        heads,
        head_bytes,
        slots.data_ptr(),
        slots.numel(),
        out.data_ptr(),
        out.stride(0) * esize,
        out.stride(1) * esize,
        dense_hs,
        chunk_tokens,
        chunk_stride,
        _native.stream_handle(stream),
    )


def gather_chunk_major(
    paged: PagedKV,
    slots: torch.Tensor,
    staging: torch.Tensor,
    *,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Gather into ``staging`` shaped [chunks, 2, chunk_tokens, *row] (contiguous).

    Each ``staging[c]`` is one stored chunk ([2, chunk_tokens, *row]) laid out
    contiguously, so the Store path moves a batch to pinned memory in one copy
    and publishes per-chunk views without a second host copy.
    """
    if staging.ndim < 3 or staging.shape[1] != 2 or not staging.is_contiguous():
        raise ValueError("chunk-major staging must be a contiguous [chunks, 2, tokens, ...] tensor")
    chunk_tokens = staging.shape[2]
    if slots.numel() != staging.shape[0] * chunk_tokens:
        raise ValueError("slot count does not fill the chunk-major staging")
    row = _row_shape(staging.shape[3:], staging.stride()[3:], staging.element_size())
    heads, head_bytes, paged_hs, dense_hs = match_rows(paged.row, row)
    esize = staging.element_size()
    _native.call(
        "cb_paged_gather",
        paged.key.data_ptr(),
        paged.value.data_ptr(),
        paged.block_stride,
        paged.slot_stride,
        paged_hs,
        paged.num_blocks,
        paged.block_size,
        heads,
        head_bytes,
        slots.data_ptr(),
        slots.numel(),
        staging.data_ptr(),
        staging.stride(1) * esize,
        staging.stride(2) * esize,
        dense_hs,
        chunk_tokens,
        staging.stride(0) * esize,
        _native.stream_handle(stream),
    )


def gather_paged_kv(
    kv_layer: KVLayer,
    slot_mapping: torch.Tensor,
    block_size: int,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Gather paged KV as contiguous ``[2, tokens, ...]`` (see module docstring)."""
    paged = describe_paged(kv_layer, block_size)
    _native.require_cuda(paged.key)
    shape = (2, int(slot_mapping.numel()), *paged.row.dims)
    if out is None:
        result = torch.empty(shape, dtype=paged.dtype, device=paged.device)
    else:
        if tuple(out.shape) != shape:
            raise ValueError(f"gather output has shape {tuple(out.shape)}, expected {shape}")
        if out.dtype != paged.dtype or out.device != paged.device:
            raise ValueError("gather output must match the KV cache dtype and device")
        result = out
    if shape[1] == 0:
        return result
    slots = device_slots(slot_mapping, paged, block_size)
    gather_into(paged, slots, result)
    return result


def scatter_paged_kv(
    contiguous: torch.Tensor,
    kv_layer: KVLayer,
    slot_mapping: torch.Tensor,
    block_size: int,
) -> None:
    """Scatter ``[2, tokens, ...]`` into a vLLM paged KV layer."""
    if contiguous.shape[0] != 2:
        raise ValueError("contiguous KV must have K/V as its first dimension")
    paged = describe_paged(kv_layer, block_size)
    _native.require_cuda(paged.key, contiguous)
    if contiguous.dtype != paged.dtype:
        raise ValueError("contiguous KV must match the KV cache dtype")
    tokens = int(slot_mapping.numel())
    if tuple(contiguous.shape) != (2, tokens, *paged.row.dims):
        raise ValueError(
            f"contiguous KV has shape {tuple(contiguous.shape)}, "
            f"expected {(2, tokens, *paged.row.dims)}"
        )
    if tokens == 0:
        return
    slots = device_slots(slot_mapping, paged, block_size)
    scatter_from(contiguous, paged, slots)


def scatter_from(
    contiguous: torch.Tensor,
    paged: PagedKV,
    slots: torch.Tensor,
    *,
    stream: torch.cuda.Stream | None = None,
) -> None:
    heads, head_bytes, paged_hs, dense_hs = match_rows(paged.row, dense_row(contiguous))
    esize = contiguous.element_size()
    _native.call(
        "cb_paged_scatter",
        contiguous.data_ptr(),
        contiguous.stride(0) * esize,
        contiguous.stride(1) * esize,
        dense_hs,
        0,
        0,
        paged.key.data_ptr(),
        paged.value.data_ptr(),
        paged.block_stride,
        paged.slot_stride,
        paged_hs,
        paged.num_blocks,
        paged.block_size,
        heads,
        head_bytes,
        slots.data_ptr(),
        slots.numel(),
        _native.stream_handle(stream),
    )


def paged_copy_error(device: torch.device | int | None = None, reset: bool = True) -> int:
    """Failure word of the bulk-copy gather/scatter kernels on ``device`` (0: none).

    Synchronizes the device's current stream.  A non-zero word means a bounded
    wait inside a launch gave up and that launch stopped early.
    """
    value = ctypes.c_int32(0)
    stream = torch.cuda.current_stream(device)
    _native.call("cb_paged_copy_error", stream.cuda_stream, ctypes.addressof(value), int(reset))
    return int(value.value)
