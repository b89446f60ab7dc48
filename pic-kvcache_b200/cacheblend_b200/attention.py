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


# exact_rounding argument -> the C ABI's mode code
_MODES = {True: 1, "reference": 1, "flash": 2, False: 0, "fused": 0}


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
    exact_rounding: bool | str = True,
) -> torch.Tensor:
    """out [Nq, Hq, D] for query [Nq, Hq, D] at ``query_positions`` (each in [0, Nk)),
    key / value [Nk, Hkv, D] (rows = positions).

    ``exact_rounding``:

    * True / ``"reference"`` -- the einsum path's roundings in its order (element-type
      logits, element-type logit * scale, the normalized probabilities rounded to the
      element type before P V): a row log2-sum-exp launch, then the products.
    * ``"flash"`` -- the same logit roundings in one launch with the unnormalized
      probabilities rounded and the row sum divided at the end (within one element-type
      ulp per probability of the reference).
    * False / ``"fused"`` -- fp32 logits * scale like the reference's fused attention
      kernel (ascend.py:814-830) and flash attention, in one launch."""
    mode = _MODES.get(exact_rounding if isinstance(exact_rounding, str) else bool(exact_rounding))
    if mode is None:
        raise ValueError(f"exact_rounding must be True, False, 'reference', 'flash' or 'fused', "
                         f"not {exact_rounding!r}")
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
        float(scale), mode, out.data_ptr(), out.stride(0) * esize,
        workspace.data_ptr(), workspace.numel(),
        0 if device_error is None else device_error.data_ptr(), _native.stream_handle(stream),
    )
    return out
