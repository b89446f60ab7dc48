"""Parity at full size, one layer's fused blend load and commit scatter, bit for
bit against the oracle, through the same C-ABI calls the bench times:

* config 2 (Qwen3-8B KV shapes): a 32,768-token request with 89 reused chunks at
  random non-contiguous positions, block_size 16;
* config 4 (Qwen3-32B KV shapes): a 65,536-token request with 192 reused chunks
  relocated from source positions anywhere in a 131,072-row RoPE table (the
  YaRN-extended context vLLM builds), so rows far past the native 40,960
  positions are relocated, not zero-filled.

Each at TP1 (8 KV heads) and as one TP8 rank's shard (1 KV head)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
import oracle

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("config,shard", [(2, 1), (2, 8), (4, 1), (4, 8)])
def test_layer_load_and_commit_vs_oracle(cuda, config, shard):
    from dataclasses import replace

    shape = replace(bench.CONFIGS[config], layers=1)
    wl = bench.Workload(shape, shard, 0, cuda, host_store=False)
    path = bench.DevicePath(wl)
    plan = wl.plan
    stream = torch.cuda.Stream(cuda)
    pages_before = _bits(wl.pages[0])
    with torch.cuda.stream(stream):
        buf = path.load_layer(0, stream)
    torch.cuda.synchronize(cuda)
    assert int(path.device_error.item()) == 0
    slots = wl.slot_mapping[: plan.allocation_end].numpy()
    table = oracle.f32_to_bf16(wl.rope.cos_sin_cache.cpu().numpy())
    hits = _bits(wl.hits[0])
    segs = [(s.source_start, s.target_start, s.length, hits[i]) for i, s in enumerate(plan.segments)]
    moved = np.full(len(segs), int(any(s.source_start != s.target_start for s in plan.segments)),
                    dtype=np.int32)
    if config == 4:  # the plan relocates chunks from far past the native 40,960 positions
        assert max(s.source_start for s in plan.segments) > 100_000
        assert table.shape[0] == 131_072
    want = oracle.blend_load(oracle.BF16, plan.allocation_end, plan.apc_prefix_tokens,
                             np.ascontiguousarray(pages_before[0]), np.ascontiguousarray(pages_before[1]),
                             slots, shape.block_size, segs, moved, table, shape.head_dim, shape.head_dim, True)
    assert np.array_equal(_bits(buf), want)

    # commit: the span of the staging back into the pages
    with torch.cuda.stream(stream):
        path.commit(0, buf, stream)
    torch.cuda.synchronize(cuda)
    k_after, v_after = np.ascontiguousarray(pages_before[0]), np.ascontiguousarray(pages_before[1])
    start = plan.apc_prefix_tokens
    oracle.paged_scatter(want[:, start:], k_after, v_after, slots[start:], shape.block_size)
    got = _bits(wl.pages[0])
    assert np.array_equal(got[0], k_after) and np.array_equal(got[1], v_after)
