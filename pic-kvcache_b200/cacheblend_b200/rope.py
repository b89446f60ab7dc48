"""RoPE relocation of cached keys and the RoPE support check.

``relocate_key`` is the drop-in for cacheblend_vllm/ascend.py:52-103.  With a
``cos_sin_cache`` it runs ``cb_relocate_key``, which evaluates the delta
rotation R(new) R(old)^-1 op by op in the key dtype exactly like the torch
expression (bit-identical output).  A rotary module without that cache is
driven through its own forward twice (inverse then forward rotation), as the
reference does; that is the model's RoPE op, not a CacheBlend kernel.
``validate_rope_support`` mirrors ascend.py:106-158.
"""

from __future__ import annotations

import weakref

import torch

from . import _native

# rotary module -> {(cache ptr, shape, dtype, device): converted table}
_tables: "weakref.WeakKeyDictionary[object, dict]" = weakref.WeakKeyDictionary()


def rope_geometry(rotary_emb) -> tuple[int, int, bool]:
    head_size = int(rotary_emb.head_size)
    rotary_dim = int(getattr(rotary_emb, "rotary_dim", head_size))
    return head_size, rotary_dim, bool(rotary_emb.is_neox_style)


def cos_sin_table(rotary_emb, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """``rotary_emb.cos_sin_cache`` converted (RNE) to the key dtype, memoised."""
    cache = rotary_emb.cos_sin_cache
    try:
        per_module = _tables.setdefault(rotary_emb, {})
    except TypeError:  # not weak-referenceable
        per_module = {}
    key = (cache.data_ptr(), tuple(cache.shape), dtype, str(device))
    table = per_module.get(key)
    if table is None:
        table = cache.to(device=device, dtype=dtype).contiguous()
        per_module.clear()
        per_module[key] = table
    return table


def _shuffle_halves(tensor: torch.Tensor, head_size: int, neox: bool) -> torch.Tensor:
    """Swap the two rotation partners of every pair (R(-x) via a forward RoPE)."""
    shape = tensor.shape
    heads = tensor.reshape(shape[0], -1, head_size)
    if neox:
        first, second = heads.chunk(2, dim=-1)
        return torch.cat((second, first), dim=-1).reshape(shape)
    return torch.stack((heads[..., 1::2], heads[..., ::2]), dim=-1).reshape(shape)


def relocate_rows(
    key: torch.Tensor,
    out: torch.Tensor,
    table: torch.Tensor,
    old_positions: torch.Tensor,
    new_positions: torch.Tensor,
    head_size: int,
    rotary_dim: int,
    neox: bool,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Launch cb_relocate_key on 2-D ``[T, heads*head_size]`` row views."""
    tokens = key.shape[0]
    width = key.shape[1]
    if width % head_size:
        raise ValueError(f"key width {width} is not a multiple of head_size {head_size}")
    if key.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("relocation rows must be contiguous")
    esize = key.element_size()
    _native.call(
        "cb_relocate_key",
        key.data_ptr(),
        out.data_ptr(),
        key.stride(0) * esize,
        out.stride(0) * esize,
        tokens,
        width // head_size,
        head_size,
        rotary_dim,
        int(neox),
        _native.dtype_code(key.dtype),
        table.data_ptr(),
        table.shape[0],
        old_positions.data_ptr(),
        new_positions.data_ptr(),
        _native.stream_handle(stream),
    )


def relocate_key(
    rotary_emb,
    old_positions: torch.Tensor,
    new_positions: torch.Tensor,
    key: torch.Tensor,
) -> torch.Tensor:
    """Move an already RoPE-encoded key from ``old`` to ``new`` positions."""
    if torch.equal(old_positions, new_positions):
        return key
    head_size, rotary_dim, neox = rope_geometry(rotary_emb)
    if not hasattr(rotary_emb, "cos_sin_cache"):
        flat = key.reshape(key.shape[0], -1)
        swapped = _shuffle_halves(flat, head_size, neox)
        _, inverse = rotary_emb(old_positions, swapped, swapped)
        restored = _shuffle_halves(inverse, head_size, neox)
        _, moved = rotary_emb(new_positions, restored, restored)
        return moved.reshape_as(key)
    _native.require_cuda(key)
    table = cos_sin_table(rotary_emb, key.dtype, key.device)
    if table.shape[-1] != rotary_dim:
        raise ValueError("RoPE cache width does not match rotary_dim")
    old = old_positions.reshape(-1).to(device=key.device, dtype=torch.long).contiguous()
    new = new_positions.reshape(-1).to(device=key.device, dtype=torch.long).contiguous()
    if old.numel() != key.shape[0] or new.numel() != key.shape[0]:
        raise ValueError("one old and one new position per key token is required")
    for positions in (old_positions, new_positions):
        if positions.device.type == "cpu" and positions.numel():
            if int(positions.min()) < 0 or int(positions.max()) >= table.shape[0]:
                raise IndexError("position outside the RoPE cos_sin_cache")
    flat = key.reshape(key.shape[0], -1)
    if flat.stride(-1) != 1:
        flat = flat.contiguous()
    out = torch.empty(flat.shape, dtype=key.dtype, device=key.device)
    relocate_rows(flat, out, table, old, new, head_size, rotary_dim, neox)
    return out.reshape(key.shape)


def validate_rope_support(model, rotary_emb) -> None:
    """Refuse RoPE variants whose relocation is not a pure delta rotation."""
    head_size = int(rotary_emb.head_size)
    rotary_dim = int(getattr(rotary_emb, "rotary_dim", head_size))
    if rotary_dim != head_size:
        raise ValueError(
            "CacheBlend requires rotary_dim == head_size; "
            f"got rotary_dim={rotary_dim}, head_size={head_size}"
        )
    model_config = getattr(model, "config", None)
    if getattr(model_config, "rope_scaling", None):
        raise ValueError("CacheBlend does not support rope_scaling")
    factor = getattr(model_config, "partial_rotary_factor", 1.0)
    factor = 1.0 if factor is None else float(factor)
    if factor != 1.0:
        raise ValueError(f"CacheBlend requires partial_rotary_factor=1.0; got {factor}")
    cache = getattr(rotary_emb, "cos_sin_cache", None)
    if not isinstance(cache, torch.Tensor) or cache.ndim != 2:
        raise ValueError("CacheBlend requires a two-dimensional RoPE cos_sin_cache")
    if cache.shape[0] == 0:
        raise ValueError("CacheBlend requires a non-empty RoPE cos_sin_cache")
    if cache.shape[-1] != rotary_dim:
        raise ValueError(
            "CacheBlend RoPE cache width does not match rotary_dim: "
            f"cache={cache.shape[-1]}, rotary_dim={rotary_dim}"
        )
    # Rows 0 and max-1 must be unit-norm rotations, otherwise R(new)R(old)^T is
    # not an inverse relocation (amplitude-scaled custom RoPE classes).
    rows = sorted({0, cache.shape[0] - 1})
    sample = cache[rows].float()
    cos, sin = sample.chunk(2, dim=-1)
    error = float((cos * cos + sin * sin - 1.0).abs().max())
    if error > 0.05:
        raise ValueError(
            f"CacheBlend requires unit-norm, unscaled RoPE; maximum sampled norm error is {error:.4f}"
        )
