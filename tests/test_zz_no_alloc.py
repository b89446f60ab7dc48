"""cb_sparse_q_scores_static: the Sparse-Q scorer for callers that cannot
allocate device memory while they score (a serving worker whose free memory
the KV cache already claimed, an FFI host holding another runtime's buffers).
Its workspace is a fixed array inside the library, so the call itself
allocates nothing.  Checked through the C ABI against cb_sparse_q_scores with a
caller-provided workspace, within the Sparse-Q tolerance (1e-3 relative), on
two calls in a row (the second reuses the array the first one left behind).
This file is collected last on purpose."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from cacheblend_b200 import _native

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def _problem(device, seed, num_keys=3000, num_queries=700, hq=16, hkv=4):
    gen = torch.Generator(device=device).manual_seed(seed)
    key = torch.randn(num_keys, hkv, 128, generator=gen, device=device).to(torch.bfloat16)
    query = torch.randn(num_queries, hq, 128, generator=gen, device=device).to(torch.bfloat16)
    rng = np.random.default_rng(seed)
    positions = np.sort(rng.choice(num_keys, size=num_queries, replace=False)).astype(np.int64)
    rows = np.arange(num_queries, dtype=np.int64)
    return query, key, torch.from_numpy(rows).to(device), torch.from_numpy(positions).to(device)


def _call(lib, name, query, key, rows, positions, scores, extra):
    status = getattr(lib, name)(
        query.data_ptr(), query.stride(0) * 2, key.data_ptr(), key.stride(0) * 2, key.shape[0],
        query.shape[1], key.shape[1], 128, 0, rows.data_ptr(), positions.data_ptr(), rows.numel(),
        ctypes.c_float(128 ** -0.5), scores.data_ptr(), *extra, _native.stream_handle(),
    )
    return status


def test_static_workspace_matches_caller_workspace(cuda):
    lib = _native.load_library()
    query, key, rows, positions = _problem(cuda, 5)
    needed = ctypes.c_int64(0)
    assert lib.cb_sparse_q_workspace_size(rows.numel(), query.shape[1], key.shape[1], 128, 0,
                                          ctypes.byref(needed)) == 0
    workspace = torch.empty(needed.value + 1024, dtype=torch.uint8, device=cuda)
    aligned = (workspace.data_ptr() + 1023) // 1024 * 1024
    expected = torch.empty(key.shape[0], dtype=torch.float32, device=cuda)
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    assert _call(lib, "cb_sparse_q_scores", query, key, rows, positions, expected,
                 (aligned, needed.value, error.data_ptr())) == 0
    torch.cuda.synchronize()
    for _ in range(2):
        got = torch.full((key.shape[0],), float("nan"), dtype=torch.float32, device=cuda)
        status = _call(lib, "cb_sparse_q_scores_static", query, key, rows, positions, got,
                       (error.data_ptr(),))
        assert status == 0, lib.cb_last_error().decode()
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), expected.cpu().numpy(), rtol=RTOL, atol=1e-6)
    assert int(error.item()) == 0


def test_static_workspace_rejects_requests_beyond_its_size(cuda):
    lib = _native.load_library()
    # 64 KV heads x 8 groups x 4,096 queries need far more than the 32 MiB array
    hkv, hq, queries = 64, 512, 4096
    needed = ctypes.c_int64(0)
    assert lib.cb_sparse_q_workspace_size(queries, hq, hkv, 128, 0, ctypes.byref(needed)) == 0
    assert needed.value > (32 << 20)
    scores = torch.empty(8, dtype=torch.float32, device=cuda)
    status = lib.cb_sparse_q_scores_static(
        None, 0, None, 0, 8, hq, hkv, 128, 0, None, None, queries, ctypes.c_float(1.0),
        scores.data_ptr(), None, _native.stream_handle(),
    )
    assert status == _native.CB_ERR_INVALID
    assert b"static workspace" in lib.cb_last_error()
