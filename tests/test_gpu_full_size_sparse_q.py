"""Sparse-Q at the full config-3 shape (Qwen3-30B-A3B, TP1 and TP2) against the
CPU oracle: 98,303 keys, 4,095 gap queries x 32 heads, the boundary score of
cacheblend_vllm/ascend.py:638-711 and the selection of ascend.py:757-796.

The oracle's outputs for these seeded inputs are in tests/golden/sparse_q_full.npz
(written by tests/golden/make_sparse_q_full.py, which runs the oracle over the
whole problem on the CPU).  Checked through the public API:
* sampled per-key scores within 1e-3 relative;
* the selected index set identical to the oracle's, except keys whose oracle
  scores tie with the top-k threshold within 1e-3 (the north-star tie rule);
* TP2: each rank scores its 2 KV heads (16 query heads), the partial scores
  are summed (the all-reduce) and selected again: the same set, same tie rule.
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from cacheblend_b200.selection import select_tokens, sparse_q_key_mass, sparse_q_scores

pytestmark = pytest.mark.gpu

RTOL = 1e-3
GOLDEN = Path(__file__).resolve().parent / "golden"


def _generator_module():
    spec = importlib.util.spec_from_file_location("make_sparse_q_full", GOLDEN / "make_sparse_q_full.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


@pytest.fixture(scope="module")
def problem(cuda):
    gen = _generator_module()
    gold = np.load(GOLDEN / "sparse_q_full.npz")
    key, queries = gen.make_inputs()
    assert [gen.checksum(key), gen.checksum(queries)] == gold["checksums"].tolist(), \
        "seeded inputs differ from the ones the fixture was made from"
    positions = gen.gap_positions()
    assert np.array_equal(positions, gold["positions"])
    query = torch.zeros(gen.KEYS, gen.Q_HEADS, gen.HEAD, dtype=torch.bfloat16, device=cuda)
    query[torch.from_numpy(positions).to(cuda)] = queries.to(cuda)
    gaps = np.zeros(gen.KEYS, dtype=bool)
    gaps[positions] = True
    return gen, gold, key.to(cuda), query, gaps, positions


def _assert_same_selection(got: np.ndarray, gold) -> None:
    want = gold["selected"].astype(np.int64)
    if np.array_equal(got, want):
        return
    swapped = np.setxor1d(got, want)
    threshold = float(gold["threshold"][0])
    band = dict(zip(gold["band_index"].tolist(), gold["band_score"].tolist()))
    outside = [int(i) for i in swapped
               if int(i) not in band or abs(band[int(i)] - threshold) > RTOL * abs(threshold)]
    assert not outside, f"{len(outside)} keys differ beyond the tie tolerance: {outside[:10]}"
    assert got.size == want.size


def test_sparse_q_full_shape_scores_and_selection(problem, cuda):
    gen, gold, key, query, gaps, positions = problem
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    scores, forced, stats = sparse_q_scores(query, key, np.arange(gen.KEYS), gaps, gen.SCALE, gen.BLOCK_SIZE,
                                            gen.OVERFLOW_BLOCKS, gen.TAIL_QUERY_TOKENS, device_error=error)
    selected = select_tokens(scores, gaps, gen.RATIO, forced).cpu().numpy()
    host = scores.cpu().numpy()
    assert int(error.item()) == 0
    assert stats["sparse_query_tokens"] == positions.size
    assert int(forced.sum()) == int(gold["forced_count"][0])
    np.testing.assert_allclose(host[::gen.SAMPLE_STRIDE], gold["sample_score"], rtol=RTOL, atol=1e-6)
    total = float(host.astype(np.float64).sum())
    assert abs(total - float(gold["total"][0])) <= RTOL * float(gold["total"][0])
    _assert_same_selection(selected, gold)


def test_sparse_q_full_shape_tp2_partial_scores(problem, cuda):
    gen, gold, key, query, gaps, positions = problem
    heads_per_rank, kv_per_rank = gen.Q_HEADS // 2, gen.KV_HEADS // 2
    total = torch.zeros(gen.KEYS, dtype=torch.float32, device=cuda)
    for rank in range(2):
        q_rank = query[:, rank * heads_per_rank:(rank + 1) * heads_per_rank].contiguous()
        k_rank = key[:, rank * kv_per_rank:(rank + 1) * kv_per_rank].contiguous()
        total += sparse_q_key_mass(q_rank, k_rank, positions, positions, gen.SCALE)
    from cacheblend_b200.selection import sparse_q_masks

    _, forced, _ = sparse_q_masks(gaps, gen.BLOCK_SIZE, gen.OVERFLOW_BLOCKS, gen.TAIL_QUERY_TOKENS)
    selected = select_tokens(total, gaps, gen.RATIO, forced).cpu().numpy()
    np.testing.assert_allclose(total.cpu().numpy()[::gen.SAMPLE_STRIDE], gold["sample_score"], rtol=RTOL,
                               atol=1e-6)
    _assert_same_selection(selected, gold)
