"""Native host fingerprints (cb_window_hashes, cb_hash_candidates) against the
exact Python polynomial hash of cacheblend_vllm/hashing.py:18-22 and numpy
membership, including token ids that wrap the 64-bit arithmetic.  CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from cacheblend_b200.matcher import TokenRangeMatcher, content_hash, hash_candidates, window_hashes


@pytest.mark.parametrize("window", [1, 7, 256])
def test_window_hashes_equal_exact_hash(window):
    rng = np.random.default_rng(window)
    tokens = rng.integers(0, 151_936, size=1500).astype(np.int64)
    tokens[[3, 500, 1499]] = [2**40 + 17, -1, 2**62]  # wrap the arithmetic
    got = window_hashes(tokens, window)
    assert got.shape == (tokens.size - window + 1,)
    for i in list(range(0, tokens.size - window + 1, 97)) + [tokens.size - window]:
        assert int(got[i]) == content_hash(tokens[i : i + window].tolist())


def test_window_hashes_short_and_invalid():
    assert window_hashes(np.arange(3), 4).size == 0
    with pytest.raises(ValueError):
        window_hashes(np.arange(3), 0)


def test_hash_candidates_match_isin():
    rng = np.random.default_rng(3)
    hashes = rng.integers(0, 2**63, size=20_000, dtype=np.int64).astype(np.uint64) * np.uint64(2)
    known = np.unique(np.concatenate([hashes[rng.choice(hashes.size, 500, replace=False)],
                                      rng.integers(0, 2**63, size=200, dtype=np.int64).astype(np.uint64)]))
    got = hash_candidates(hashes, known)
    assert np.array_equal(got, np.flatnonzero(np.isin(hashes, known)))
    assert hash_candidates(hashes, known[:0]).size == 0
    # more candidates than the first output buffer holds
    many = np.unique(hashes)
    assert np.array_equal(hash_candidates(hashes, many), np.arange(hashes.size))


def test_match_is_leftmost_greedy_with_verification():
    m = TokenRangeMatcher(4)
    prompt = [9, 1, 2, 3, 4, 1, 2, 3, 4, 5, 6, 7, 8]
    for record in m.make_records("s", 1, prompt, 2):  # chunks [1,2,3,4] and [1,2,3,4]... at 1 and 5
        m.register(record)
    segs = m.match("s", prompt, 0)
    assert [seg.target_start for seg in segs] == [1, 5]
    # same hash, different tokens: a forged record of the same id never matches
    assert m.match("s", [1, 2, 3, 5], 0) == ()
    assert m.match("other", prompt, 0) == ()
