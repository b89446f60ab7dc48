"""Failure detection without a GPU fault: every bounded wait the pipelined
kernels use gives up on a barrier that never completes, reports into the
caller's error word and returns, and the context keeps working."""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200 import _native
from cacheblend_b200.kv_layout import gather_paged_kv

pytestmark = pytest.mark.gpu


def test_bounded_waits_give_up_and_report(cuda):
    result = torch.zeros(1, dtype=torch.int32, device=cuda)
    start = time.perf_counter()
    _native.call("cb_wait_selftest", result.data_ptr(), _native.stream_handle())
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    assert int(result.item()) == 0b1111  # all four helpers timed out and said so
    assert 1.5 < elapsed < 60  # bounded by the 2 s limit, not a hang
    # the context still runs the hot path correctly afterwards
    rng = np.random.default_rng(1)
    kv = rng.integers(0, 1 << 16, size=(2, 8, 4, 2, 16), dtype=np.uint16)
    slots = np.array([3, 9, 17, 30], dtype=np.int64)
    t = torch.from_numpy(kv.view(np.int16)).view(torch.bfloat16).to(cuda)
    got = gather_paged_kv((t[0], t[1]), torch.from_numpy(slots).to(cuda), 4)
    want = oracle.paged_gather(np.ascontiguousarray(kv[0]), np.ascontiguousarray(kv[1]), slots, 4)
    assert np.array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16), want)
