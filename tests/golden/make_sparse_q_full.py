"""Full-size Sparse-Q fixture (config 3 at TP1): tests/golden/sparse_q_full.npz.

Qwen3-30B-A3B shapes: a 98,304-token prompt whose last token stays with vLLM
(98,303 keys, 4 KV heads, 32 query heads, head_dim 128, bf16); 16 gap chunks
of 256 tokens, the trailing one among them, act as the 4,095 sparse queries;
scale 1/sqrt(128); block_size 16, overflow_blocks 1, tail_query_tokens 64,
recompute ratio 0.15.  Inputs are N(0, 1) from a seeded CPU torch generator
(regenerated bit for bit by the GPU test, which checks their checksums first).

The expected outputs come from the CPU oracle (oracle.sparse_q_key_mass, the
restatement of cacheblend_vllm/ascend.py:638-711, pinned to the reference's
own vectors by tests/test_oracle_golden.py) and oracle.select
(ascend.py:757-796), computed in worker processes over query chunks and summed
in float64.  Stored: the selected index set, the top-k threshold, every
candidate whose score lies within 2e-3 of the threshold (the ties the test
may swap), a strided sample of the per-key scores and their total.

    python tests/golden/make_sparse_q_full.py [--workers N]
"""

from __future__ import annotations

import argparse
import multiprocessing as mp
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
OUT = HERE / "sparse_q_full.npz"

KEYS = 98_303
Q_HEADS, KV_HEADS, HEAD = 32, 4, 128
CHUNK, GAP_CHUNKS = 256, 16
BLOCK_SIZE, OVERFLOW_BLOCKS, TAIL_QUERY_TOKENS, RATIO = 16, 1, 64, 0.15
SCALE = 128 ** -0.5
INPUT_SEED, PLAN_SEED = 303, 3
SAMPLE_STRIDE = 61
TIE_BAND = 2e-3


def gap_positions() -> np.ndarray:
    """15 seeded gap chunks plus the trailing partial chunk (the last prompt token excluded)."""
    rng = np.random.default_rng(PLAN_SEED)
    full_chunks = KEYS // CHUNK
    chosen = rng.choice(full_chunks, size=GAP_CHUNKS - 1, replace=False)
    parts = [c * CHUNK + np.arange(CHUNK) for c in chosen] + [np.arange(full_chunks * CHUNK, KEYS)]
    return np.sort(np.concatenate(parts)).astype(np.int64)


def make_inputs():
    """(key [KEYS, 4, 128], sparse queries [Q, 32, 128]) as bf16 torch tensors on the CPU."""
    import torch

    gen = torch.Generator().manual_seed(INPUT_SEED)
    key = torch.randn(KEYS, KV_HEADS, HEAD, generator=gen).to(torch.bfloat16)
    queries = torch.randn(gap_positions().size, Q_HEADS, HEAD, generator=gen).to(torch.bfloat16)
    return key, queries


def checksum(tensor) -> int:
    """Sum of the 16-bit patterns (detects any change of the seeded inputs)."""
    import torch

    return int(tensor.view(torch.int16).to(torch.int64).sum())


def _mass_of_chunks(args):
    start, stop = args
    sys.path.insert(0, str(REPO))
    import oracle

    key, queries = make_inputs()
    positions = gap_positions()
    return oracle.sparse_q_key_mass(queries[start:stop].float().numpy(), key.float().numpy(),
                                    positions[start:stop], SCALE)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--workers", type=int, default=os.cpu_count() or 1)
    args = parser.parse_args()
    sys.path.insert(0, str(REPO))
    import oracle

    positions = gap_positions()
    # query slices that keep the oracle's chunks of 8 intact
    bounds = np.linspace(0, positions.size // 8, 4 * args.workers + 1).astype(int) * 8
    bounds[-1] = positions.size
    jobs = [(int(a), int(b)) for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
    began = time.time()
    with mp.get_context("spawn").Pool(args.workers) as pool:
        mass = np.sum(pool.map(_mass_of_chunks, jobs), axis=0)
    scores = mass.astype(np.float32)
    gaps = np.zeros(KEYS, dtype=bool)
    gaps[positions] = True
    _, forced, _ = oracle.sparse_q_masks(gaps, BLOCK_SIZE, OVERFLOW_BLOCKS, TAIL_QUERY_TOKENS)
    selected = oracle.select(scores, gaps, RATIO, forced)
    base = gaps | forced
    candidates = np.flatnonzero(~base)
    k = selected.size - int(base.sum())
    threshold = np.float32(np.sort(scores[candidates])[::-1][k - 1])
    band = candidates[np.abs(scores[candidates] - threshold) <= TIE_BAND * abs(threshold)]
    sample = np.arange(0, KEYS, SAMPLE_STRIDE)
    key, queries = make_inputs()
    np.savez_compressed(
        OUT,
        meta=np.array([KEYS, Q_HEADS, KV_HEADS, HEAD, INPUT_SEED, PLAN_SEED, SAMPLE_STRIDE], dtype=np.int64),
        checksums=np.array([checksum(key), checksum(queries)], dtype=np.int64),
        positions=positions.astype(np.int32),
        selected=selected.astype(np.int32),
        forced_count=np.array([int(forced.sum())], dtype=np.int64),
        threshold=np.array([threshold], dtype=np.float32),
        band_index=band.astype(np.int32),
        band_score=scores[band],
        sample_score=scores[sample],
        total=np.array([float(mass.sum())], dtype=np.float64),
    )
    print(f"{OUT.name}: {selected.size} selected (k={k}), threshold {threshold:.6g}, "
          f"{band.size} within the tie band, oracle {time.time() - began:.0f} s on {args.workers} workers")


if __name__ == "__main__":
    main()
