"""The fused K-deviation + selection launch (cb_kv_deviation_select) of a
single-rank check layer: the deviation expression and ``_select`` of
cacheblend_vllm/ascend.py:534-543 and 757-796 in one kernel.  Its scores must
equal the oracle's bit for bit (same association order as cb_kv_deviation) and
its index set the oracle's select exactly (ties: lowest index; NaN above +inf),
on the warp-per-token rows, the packed small rows, the fallback shapes
(unaligned rows, more tokens than one cluster holds), with every gap (k = 0),
with ties, with out-of-range cached rows, on calls back to back (the workspace
is left zeroed by each call) and replayed from a CUDA graph."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.selection import deviation_select, kv_deviation, select_tokens

pytestmark = pytest.mark.gpu

CODES = {torch.bfloat16: oracle.BF16, torch.float16: oracle.FP16, torch.float32: oracle.FP32}


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float32:
        return t.numpy()
    if t.dtype == torch.float16:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def _case(cuda, n, width, dtype, seed, offset=300, gap_fraction=0.2):
    gen = torch.Generator(device=cuda).manual_seed(seed)
    total = n + offset + 50
    cached = torch.randn(total, width, generator=gen, device=cuda).to(dtype)
    fresh = (cached[offset:offset + n].float() + 0.05 * torch.randn(n, width, generator=gen, device=cuda)).to(dtype)
    gaps = np.random.default_rng(seed).random(n) < gap_fraction
    return fresh, cached, gaps


def _expect(fresh, cached, gaps, ratio, offset=0, index=None):
    code = CODES[fresh.dtype]
    scores = oracle.kv_deviation(bits(fresh), bits(cached), code, abs_index=index, abs_offset=offset)
    return scores, oracle.select(scores, gaps, ratio)


@pytest.mark.parametrize("n,width,dtype", [
    (4096, 1024, torch.bfloat16),     # 8 heads: a warp per token
    (32768, 128, torch.bfloat16),     # one head (a TP8 rank): tokens packed per warp
    (1000, 256, torch.float16),       # two heads, fp16
    (2500, 256, torch.float32),       # fp32 rows
    (777, 100, torch.bfloat16),       # rows not 16-byte aligned: the two-launch fallback
    (400_000, 8, torch.bfloat16),     # more tokens than one cluster holds: the fallback
    (5, 1024, torch.bfloat16),        # fewer tokens than a cluster has CTAs
])
def test_fused_matches_oracle(cuda, n, width, dtype):
    fresh, cached, gaps = _case(cuda, n, width, dtype, n + width)
    selected, scores = deviation_select(fresh, cached, gaps, 0.15, absolute_offset=300)
    want_scores, want_sel = _expect(fresh, cached, gaps, 0.15, offset=300)
    assert np.array_equal(scores.cpu().numpy(), want_scores)
    assert np.array_equal(selected.cpu().numpy(), want_sel)
    # and the same as the two-launch path
    two = select_tokens(kv_deviation(fresh, cached, absolute_offset=300), gaps, 0.15).cpu().numpy()
    assert np.array_equal(selected.cpu().numpy(), two)


def test_fused_back_to_back_calls_and_edge_masks(cuda):
    fresh, cached, gaps = _case(cuda, 20_000, 1024, torch.bfloat16, 3)
    first = [t.cpu().numpy() for t in deviation_select(fresh, cached, gaps, 0.15, absolute_offset=300)]
    for _ in range(3):  # the workspace's histogram and ticket start at zero again every time
        again = [t.cpu().numpy() for t in deviation_select(fresh, cached, gaps, 0.15, absolute_offset=300)]
        assert all(np.array_equal(a, b) for a, b in zip(first, again))
    # every token a gap: k = 0, the gaps alone
    all_gaps = np.ones(20_000, dtype=bool)
    sel, _ = deviation_select(fresh, cached, all_gaps, 0.15, absolute_offset=300)
    assert np.array_equal(sel.cpu().numpy(), np.arange(20_000))
    # no gap at all
    none = np.zeros(20_000, dtype=bool)
    sel, scores = deviation_select(fresh, cached, none, 0.15, absolute_offset=300)
    assert np.array_equal(sel.cpu().numpy(), oracle.select(scores.cpu().numpy(), none, 0.15))


def test_fused_ties_keep_the_lowest_indices(cuda):
    gen = torch.Generator(device=cuda).manual_seed(9)
    cached = torch.randn(5000, 256, generator=gen, device=cuda).to(torch.bfloat16)
    fresh = cached.clone()
    fresh[::7] += 1.0  # a seventh of the rows deviate by the same amount: exact ties
    gaps = np.zeros(5000, dtype=bool)
    gaps[100:200] = True
    sel, scores = deviation_select(fresh, cached, gaps, 0.05)
    want = oracle.select(scores.cpu().numpy(), gaps, 0.05)
    assert np.array_equal(sel.cpu().numpy(), want)


def test_fused_out_of_range_rows_rank_first(cuda):
    gen = torch.Generator(device=cuda).manual_seed(13)
    cached = torch.randn(3000, 256, generator=gen, device=cuda).to(torch.bfloat16)
    fresh = torch.randn(2000, 256, generator=gen, device=cuda).to(torch.bfloat16)
    index = torch.arange(2000, dtype=torch.int64)
    index[[4, 900, 1999]] = torch.tensor([-3, 3000, 10**9])
    gaps = np.zeros(2000, dtype=bool)
    sel, scores = deviation_select(fresh, cached, gaps, 0.1, absolute_indices=index)
    got = scores.cpu().numpy()
    assert np.isnan(got[[4, 900, 1999]]).all()
    assert np.array_equal(sel.cpu().numpy(), oracle.select(got, gaps, 0.1))
    assert {4, 900, 1999} <= set(sel.cpu().numpy().tolist())


def test_fused_graph_replay_equals_eager(cuda):
    fresh, cached, gaps = _case(cuda, 8192, 1024, torch.bfloat16, 21)
    eager, eager_scores = deviation_select(fresh, cached, gaps, 0.15, absolute_offset=300)
    base = torch.from_numpy(gaps.astype(np.uint8)).to(cuda)
    stream = torch.cuda.Stream(cuda)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        captured, captured_scores = deviation_select(fresh, cached, gaps, 0.15, absolute_offset=300,
                                                     stream=stream, base_mask_device=base)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(captured, eager) and torch.equal(captured_scores, eager_scores)
