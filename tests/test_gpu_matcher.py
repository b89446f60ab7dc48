"""The native host fingerprints (cb_window_hashes, cb_hash_candidates) on the GPU
box: the scheduler-side lookup runs there in production (vLLM's scheduler
process, no CUDA context), so the GPU session also checks it against the
reference's own fingerprints (tests/golden/hashes.npz, from
cacheblend_vllm/hashing.py:18-53) and runs one Sparse-Q-sized lookup
(matcher.py:80-125) end to end."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from cacheblend_b200.matcher import TokenRangeMatcher, chunk_hashes, content_hash, window_hashes

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "hashes.npz"


def test_fingerprints_equal_reference_vectors_on_the_box(cuda):
    gold = np.load(GOLDEN)
    tokens = gold["tokens"]
    assert np.array_equal(window_hashes(tokens, 256), gold["windows"])
    assert np.array_equal(chunk_hashes(tokens.reshape(16, 256)), gold["chunks"])
    assert [content_hash([7]), content_hash([-1, 0, 1]), content_hash([])] == gold["small"].tolist()


def test_long_prompt_lookup_finds_every_registered_chunk(cuda):
    """98,304-token prompt: 80 % of its 384 chunks were stored from another
    request at other offsets; the match must return each at its own target."""
    rng = np.random.default_rng(77)
    chunk = 256
    prompt = rng.integers(0, 151_936, size=98_304).astype(np.int64)
    reused = np.sort(rng.choice(384, size=307, replace=False))
    matcher = TokenRangeMatcher(chunk)
    for i, c in enumerate(reused):
        tokens = prompt[c * chunk:(c + 1) * chunk].tolist()
        matcher.register(matcher.make_record("scope", 5_000 + i * chunk, tokens))
    segments = matcher.match("scope", prompt.tolist(), 0)
    assert [seg.target_start for seg in segments] == [int(c) * chunk for c in reused]
    assert all(seg.segment_id.source_start == 5_000 + i * chunk for i, seg in enumerate(segments))
