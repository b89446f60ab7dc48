"""cb_sparse_q_scores_static: the Sparse-Q scorer for callers that cannot
allocate device memory while they score -- a serving worker whose free memory
the KV cache already claimed after profiling, or an FFI host holding another
runtime's buffers without an allocator of its own.  Its workspace is a fixed
array inside the library, so the call itself allocates nothing.

Checked through the C ABI, for bf16 and fp16, on two calls in a row (the second
reuses the array the first one left behind): against cb_sparse_q_scores with a
caller-provided workspace and against the CPU oracle, within the Sparse-Q
tolerance (1e-3 relative); and that neither torch's allocator nor the device's
free memory changes across the calls.  This file is collected last on purpose,
and passes alone in a fresh process as well as after the other tests."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200 import _native

pytestmark = pytest.mark.gpu

RTOL = 1e-3
ATOL = 1e-6
DTYPES = {0: torch.bfloat16, 1: torch.float16}


def _problem(device, seed, dtype_code, num_keys=3000, num_queries=700, hq=16, hkv=4):
    gen = torch.Generator().manual_seed(seed)
    dtype = DTYPES[dtype_code]
    key = torch.randn(num_keys, hkv, 128, generator=gen).to(dtype)
    query = torch.randn(num_queries, hq, 128, generator=gen).to(dtype)
    rng = np.random.default_rng(seed)
    positions = np.sort(rng.choice(num_keys, size=num_queries, replace=False)).astype(np.int64)
    rows = np.arange(num_queries, dtype=np.int64)
    return (query.to(device), key.to(device), torch.from_numpy(rows).to(device),
            torch.from_numpy(positions).to(device), query.float().numpy(), key.float().numpy(), positions)


def _call(lib, name, query, key, rows, positions, scores, dtype_code, extra):
    return getattr(lib, name)(
        query.data_ptr(), query.stride(0) * 2, query.shape[0], key.data_ptr(), key.stride(0) * 2,
        key.shape[0], query.shape[1], key.shape[1], 128, dtype_code, rows.data_ptr(),
        positions.data_ptr(), rows.numel(), ctypes.c_float(128 ** -0.5), scores.data_ptr(), *extra,
        _native.stream_handle(),
    )


@pytest.mark.parametrize("dtype_code", [0, 1], ids=["bf16", "fp16"])
def test_static_workspace_matches_caller_workspace_and_oracle(cuda, dtype_code):
    lib = _native.load_library()
    query, key, rows, positions, q_host, k_host, pos_host = _problem(cuda, 5 + dtype_code, dtype_code)
    needed = ctypes.c_int64(0)
    assert lib.cb_sparse_q_workspace_size(rows.numel(), query.shape[1], key.shape[1], 128, dtype_code,
                                          ctypes.byref(needed)) == 0
    workspace = torch.empty(needed.value + 1024, dtype=torch.uint8, device=cuda)
    aligned = (workspace.data_ptr() + 1023) // 1024 * 1024
    expected = torch.empty(key.shape[0], dtype=torch.float32, device=cuda)
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    assert _call(lib, "cb_sparse_q_scores", query, key, rows, positions, expected, dtype_code,
                 (aligned, needed.value, error.data_ptr())) == 0
    torch.cuda.synchronize()
    want = oracle.sparse_q_key_mass(q_host, k_host, pos_host, 128 ** -0.5,
                                    dtype=dtype_code).astype(np.float32)
    outputs = [torch.full((key.shape[0],), float("nan"), dtype=torch.float32, device=cuda)
               for _ in range(2)]
    status = _call(lib, "cb_sparse_q_scores_static", query, key, rows, positions, outputs[0], dtype_code,
                   (error.data_ptr(),))
    assert status == 0, lib.cb_last_error().decode()
    torch.cuda.synchronize()
    # the first call set the array up; the second allocates nothing anywhere
    allocated = torch.cuda.memory_allocated(cuda)
    free_before, _ = torch.cuda.mem_get_info(cuda)
    status = _call(lib, "cb_sparse_q_scores_static", query, key, rows, positions, outputs[1], dtype_code,
                   (error.data_ptr(),))
    assert status == 0, lib.cb_last_error().decode()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(cuda)
    assert torch.cuda.memory_allocated(cuda) == allocated
    assert free_after == free_before
    assert int(error.item()) == 0
    for got in outputs:
        got = got.cpu().numpy()
        np.testing.assert_allclose(got, expected.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_static_workspace_rejects_requests_beyond_its_size(cuda):
    lib = _native.load_library()
    # 64 KV heads x 8 groups x 4,096 queries need far more than the 32 MiB array
    hkv, hq, queries = 64, 512, 4096
    needed = ctypes.c_int64(0)
    assert lib.cb_sparse_q_workspace_size(queries, hq, hkv, 128, 0, ctypes.byref(needed)) == 0
    assert needed.value > (32 << 20)
    scores = torch.empty(8, dtype=torch.float32, device=cuda)
    status = lib.cb_sparse_q_scores_static(
        None, 0, 0, None, 0, 8, hq, hkv, 128, 0, None, None, queries, ctypes.c_float(1.0),
        scores.data_ptr(), None, _native.stream_handle(),
    )
    assert status == _native.CB_ERR_INVALID
    assert b"static workspace" in lib.cb_last_error()
    # a query count whose size arithmetic would overflow is refused before any sizing
    status = lib.cb_sparse_q_scores_static(
        None, 0, 0, None, 0, 8, hq, hkv, 128, 0, None, None, 1 << 40, ctypes.c_float(1.0),
        scores.data_ptr(), None, _native.stream_handle(),
    )
    assert status == _native.CB_ERR_INVALID
    assert b"too many queries" in lib.cb_last_error()
