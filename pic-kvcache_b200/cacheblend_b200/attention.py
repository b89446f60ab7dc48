"""Blend attention on the tensor cores (cb_blend_attention).

The side executor's attention of the computed, possibly pruned, queries over
the whole staging context: Qwen3BlendExecutor._attention
(cacheblend_vllm/ascend.py:798-846).  Queries sit at absolute positions and
attend every staging row at or before their position; grouped query heads
share their KV head.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native


def attention_supported(query: torch.Tensor, key: torch.Tensor) -> bool:
    """Shapes cb_blend_attention takes: head size 128, bf16 / fp16, query heads
    a multiple of KV heads with the group count dividing 128."""
    if query.ndim != 3 or key.ndim != 3 or query.shape[2] != 128 or key.shape[2] != 128:
        return False
    if query.dtype not in (torch.bfloat16, torch.float16) or key.dtype != query.dtype:
        return False
    hq, hkv = query.shape[1], key.shape[1]
    return hkv > 0 and hq % hkv == 0 and 128 % (hq // hkv) == 0


def attention_workspace_bytes(num_queries: int, num_keys: int, num_q_heads: int, num_kv_heads: int,
                              head_size: int, dtype: torch.dtype) -> int:
    out = ctypes.c_int64(0)
    _native.call("cb_blend_attention_workspace_size", num_queries, num_keys, num_q_heads,
                 num_kv_heads, head_size, _native.dtype_code(dtype), ctypes.addressof(out))
    return int(out.value)


def blend_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    query_positions: torch.Tensor,
    scale: float,
    workspace: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
    exact_rounding: bool = True,
) -> torch.Tensor:
    """out [Nq, Hq, D] for query [Nq, Hq, D] at ``query_positions`` (each in [0, Nk)),
    key / value [Nk, Hkv, D] (rows = positions).

    ``exact_rounding`` keeps the einsum path's roundings (element-type logits, element-type
    logit * scale); False computes fp32 logits * scale like the reference's fused attention
    kernel (ascend.py:814-830) and flash attention, about a fifth faster."""
    _native.require_cuda(query, key, value)
    if query.ndim != 3 or key.ndim != 3 or value.shape != key.shape:
        raise ValueError("query must be [tokens, q_heads, head]; key and value [keys, kv_heads, head]")
    if not (query.dtype == key.dtype == value.dtype):
        raise ValueError("query, key and value must share a dtype")
    for name, t in (("query", query), ("key", key), ("value", value)):
        if t.stride(2) != 1 or t.stride(1) != t.shape[2]:
            raise ValueError(f"{name} heads must be contiguous within a row")
    num_queries, num_q_heads, head_size = query.shape
    num_keys, num_kv_heads, _ = key.shape
    positions = query_positions.to(device=query.device, dtype=torch.long).contiguous()
    if positions.numel() != num_queries:
        raise ValueError("one position per query row is required")
    out = torch.empty_like(query, memory_format=torch.contiguous_format)
    if num_queries == 0:
        return out
    need = attention_workspace_bytes(num_queries, num_keys, num_q_heads, num_kv_heads, head_size,
                                     query.dtype)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=query.device)
    esize = query.element_size()
    _native.call(
        "cb_blend_attention", query.data_ptr(), query.stride(0) * esize, key.data_ptr(),
        key.stride(0) * esize, value.data_ptr(), value.stride(0) * esize, num_keys, num_q_heads,
        num_kv_heads, head_size, _native.dtype_code(query.dtype), positions.data_ptr(), num_queries,
        float(scale), int(bool(exact_rounding)), out.data_ptr(), out.stride(0) * esize,
        workspace.data_ptr(), workspace.numel(),
        0 if device_error is None else device_error.data_ptr(), _native.stream_handle(stream),
    )
    return out
