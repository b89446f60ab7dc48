"""Tensor-parallel score semantics on one GPU: every rank scores its share of
the KV heads and the ranks' fp32 scores are all-reduced (summed) before the
select (cacheblend_vllm/ascend.py:764-770).  The sum of the per-shard scores
must equal the single-rank score over all heads (fp32 summation order aside),
and the selection made from it must be the same."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cacheblend_b200.selection import kv_deviation, select_tokens, sparse_q_key_mass

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_deviation_shards_sum_to_full(cuda, tp):
    gen = torch.Generator(device=cuda).manual_seed(tp)
    heads, hd, n, total = 8, 128, 4096, 5000
    cached = torch.randn(total, heads, hd, generator=gen, device=cuda).to(torch.bfloat16)
    fresh = (cached[900 : 900 + n].float() + 0.05 * torch.randn(n, heads, hd, generator=gen, device=cuda)).to(
        torch.bfloat16)
    full = kv_deviation(fresh.reshape(n, -1), cached.reshape(total, -1), absolute_offset=900)
    per = heads // tp
    parts = [kv_deviation(fresh[:, r * per : (r + 1) * per].reshape(n, -1).contiguous(),
                          cached[:, r * per : (r + 1) * per].reshape(total, -1).contiguous(),
                          absolute_offset=900) for r in range(tp)]
    reduced = torch.stack(parts).sum(0)
    torch.testing.assert_close(reduced, full, rtol=2e-6, atol=0)
    gaps = np.zeros(n, dtype=bool)
    gaps[::17] = True
    a = select_tokens(full, gaps, 0.15).cpu().numpy()
    b = select_tokens(reduced, gaps, 0.15).cpu().numpy()
    # identical unless two scores straddle the threshold within the summation error
    assert len(a) == len(b) and len(np.setxor1d(a, b)) <= 2


@pytest.mark.parametrize("tp", [2, 4])
def test_sparse_q_shards_sum_to_full(cuda, tp):
    gen = torch.Generator(device=cuda).manual_seed(40 + tp)
    hq, hkv, hd, ctx = 32, 4, 128, 3000
    query = torch.randn(ctx, hq, hd, generator=gen, device=cuda).to(torch.bfloat16)
    key = torch.randn(ctx, hkv, hd, generator=gen, device=cuda).to(torch.bfloat16)
    positions = np.sort(np.concatenate([np.arange(600, 856), np.arange(2000, 2100), [ctx - 1]]))
    rows = positions
    scale = hd ** -0.5
    full = sparse_q_key_mass(query, key, rows, positions, scale)
    qper, kper = hq // tp, hkv // tp
    parts = [sparse_q_key_mass(query[:, r * qper : (r + 1) * qper].contiguous(),
                               key[:, r * kper : (r + 1) * kper].contiguous(), rows, positions, scale)
             for r in range(tp)]
    reduced = torch.stack(parts).sum(0)
    torch.testing.assert_close(reduced, full, rtol=1e-5, atol=1e-7)
