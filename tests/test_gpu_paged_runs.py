"""Paged gather/scatter over block runs (the bulk-copy kernel used when rows are
contiguous on both sides) against the oracle, bit for bit: spans starting
mid-block, every block size from 1 to 128, rows from 16 B to 34 KiB, slots
that wrap or fall out of range, non-run slot orders, and the chunk-major Store
staging.  Every case also checks the kernels' failure word stays clear."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.kv_layout import (
    describe_paged, gather_chunk_major, gather_paged_kv, paged_copy_error, scatter_paged_kv,
)

pytestmark = pytest.mark.gpu


def _bf16(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _case(rng, bs, heads, hd, tokens, shuffle_runs):
    nb = max(4, (tokens + 2 * bs - 1) // bs + 3)
    k = rng.integers(0, 1 << 16, size=(nb, bs, heads, hd), dtype=np.uint16) & 0xBFFF
    v = rng.integers(0, 1 << 16, size=(nb, bs, heads, hd), dtype=np.uint16) & 0xBFFF
    blocks = rng.permutation(nb)
    start = int(rng.integers(0, bs))
    slots = np.array([blocks[(start + t) // bs] * bs + (start + t) % bs for t in range(tokens)],
                     dtype=np.int64)
    if shuffle_runs and tokens > 8:
        idx = rng.permutation(tokens)[: tokens // 3]
        slots[np.sort(idx)] = slots[idx]  # breaks runs, keeps slots distinct
    return k, v, slots, nb


@pytest.mark.parametrize("bs", [1, 16, 32, 128])
@pytest.mark.parametrize("heads,hd", [(1, 8), (1, 128), (8, 128), (136, 128)])
@pytest.mark.parametrize("tokens", [1, 37, 1000])
def test_gather_scatter_runs_vs_oracle(cuda, bs, heads, hd, tokens):
    rng = np.random.default_rng(bs * 1000 + heads * 10 + tokens)
    for shuffle in (False, True):
        k, v, slots, nb = _case(rng, bs, heads, hd, tokens, shuffle)
        cache = torch.stack([_bf16(k, cuda), _bf16(v, cuda)])
        got = gather_paged_kv(cache, torch.from_numpy(slots), bs)
        assert np.array_equal(_bits(got), oracle.paged_gather(k, v, slots, bs))
        src = rng.integers(0, 1 << 16, size=(2, tokens, heads, hd), dtype=np.uint16) & 0xBFFF
        scatter_paged_kv(_bf16(src, cuda), cache, torch.from_numpy(slots), bs)
        k2, v2 = k.copy(), v.copy()
        oracle.paged_scatter(src, k2, v2, slots, bs)
        assert np.array_equal(_bits(cache[0]), k2) and np.array_equal(_bits(cache[1]), v2)
    assert paged_copy_error(cuda) == 0


def test_wrapped_and_out_of_range_slots(cuda):
    rng = np.random.default_rng(5)
    k, v, slots, nb = _case(rng, 16, 8, 128, 300, False)
    slots[1] = -1  # torch wrap: the last slot of the pool
    slots[2] = nb * 16 + 5  # out of range: the kernel skips the row
    cache = torch.stack([_bf16(k, cuda), _bf16(v, cuda)])
    out = torch.zeros(2, 300, 8, 128, dtype=torch.bfloat16, device=cuda)
    from cacheblend_b200.kv_layout import gather_into

    gather_into(describe_paged(cache, 16), torch.from_numpy(slots).to(cuda), out)
    want = np.zeros((2, 300, 8, 128), dtype=np.uint16)
    ok = np.arange(300) != 2
    want[:, ok] = oracle.paged_gather(k, v, slots[ok], 16)
    assert np.array_equal(_bits(out), want)
    assert paged_copy_error(cuda) == 0


@pytest.mark.parametrize("start", [0, 5])
def test_chunk_major_gather_vs_oracle(cuda, start):
    rng = np.random.default_rng(9 + start)
    bs, heads, hd, chunk, chunks = 16, 8, 128, 256, 3
    k, v, slots, nb = _case(rng, bs, heads, hd, chunks * chunk + start, False)
    slots = slots[start:]
    cache = torch.stack([_bf16(k, cuda), _bf16(v, cuda)])
    staging = torch.empty(chunks, 2, chunk, heads, hd, dtype=torch.bfloat16, device=cuda)
    gather_chunk_major(describe_paged(cache, bs), torch.from_numpy(slots).to(cuda), staging)
    want = oracle.paged_gather(k, v, slots, bs)
    for c in range(chunks):
        assert np.array_equal(_bits(staging[c]), want[:, c * chunk : (c + 1) * chunk])
    assert paged_copy_error(cuda) == 0
