"""Sparse-Q scorer on the tcgen05 tensor cores vs the reference's golden
vectors and the CPU oracle.  Scores: within 1e-3 relative (fp32); selected
index sets: identical, except entries whose scores tie with the top-k
threshold within that tolerance."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.selection import select_tokens, sparse_q_key_mass, sparse_q_scores

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def _bf16(bits, device):
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def _check_selection(got_sel, got_scores, want_scores, gaps, forced, ratio=0.15):
    """Index sets equal, or differing only where scores tie at the threshold within RTOL."""
    want_sel = oracle.select(want_scores, gaps, ratio, forced)
    if np.array_equal(got_sel, want_sel):
        return
    diff = np.setxor1d(got_sel, want_sel)
    base = gaps | forced
    candidates = np.flatnonzero(~base)
    k = len(want_sel) - int(base.sum())
    threshold = np.sort(want_scores[candidates])[::-1][k - 1]
    assert np.all(np.abs(want_scores[diff] - threshold) <= RTOL * abs(threshold)), diff


@pytest.mark.parametrize("case", range(2))
def test_sparse_q_golden(golden, cuda, case):
    tag = f"sq128_{case}"
    chunk, overflow, tail, block_size = (int(x) for x in golden[f"{tag}_meta"])
    query = _bf16(golden[f"{tag}_query"], cuda)
    key = _bf16(golden[f"{tag}_key"], cuda)
    gaps = golden[f"{tag}_gaps"]
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    scores, forced, stats = sparse_q_scores(query, key, golden[f"{tag}_absolute"], gaps,
                                            float(golden[f"{tag}_scale"][0]), block_size, overflow, tail,
                                            device_error=error)
    got = scores.cpu().numpy()
    np.testing.assert_allclose(got, golden[f"{tag}_scores"], rtol=RTOL, atol=1e-6)
    assert int(error.item()) == 0
    assert np.array_equal(forced.cpu().numpy(), golden[f"{tag}_forced"])
    assert stats["sparse_query_tokens"] == golden[f"{tag}_stats"][0]
    sel = select_tokens(scores, gaps, 0.15, forced.cpu().numpy()).cpu().numpy()
    _check_selection(sel, got, golden[f"{tag}_scores"], gaps, golden[f"{tag}_forced"])


@pytest.mark.parametrize("hq,hkv,dtype", [(32, 4, torch.bfloat16), (16, 8, torch.bfloat16),
                                          (8, 1, torch.float16), (64, 8, torch.bfloat16)])
def test_sparse_q_vs_oracle_mid_size(cuda, hq, hkv, dtype):
    gen = torch.Generator(device=cuda).manual_seed(hq * 10 + hkv)
    ctx, active = 2300, 1900
    query = torch.randn(active, hq, 128, generator=gen, device=cuda).to(dtype)
    key = torch.randn(ctx, hkv, 128, generator=gen, device=cuda).to(dtype)
    absolute = np.arange(ctx - active, ctx)
    gaps = np.zeros(active, dtype=bool)
    gaps[300:556] = True
    gaps[1600:1700] = True
    gaps[-1] = True
    scale = 128 ** -0.5
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    scores, forced, _ = sparse_q_scores(query, key, absolute, gaps, scale, 16, 1, 64, device_error=error)
    assert int(error.item()) == 0
    to_f = (lambda t: t.float().cpu().numpy())
    want, want_forced, _ = oracle.sparse_q_scores(to_f(query), to_f(key), absolute, gaps, scale, 16, 1, 64)
    got = scores.cpu().numpy()
    if dtype == torch.bfloat16:
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=1e-6)
        _check_selection(select_tokens(scores, gaps, 0.15, want_forced).cpu().numpy(), got, want, gaps,
                         want_forced)
    else:
        # fp16 logits round to fp16 (reference: the matmul output dtype); the bf16
        # oracle differs by that rounding only, far inside 1e-2
        np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-5)
    assert np.array_equal(forced.cpu().numpy(), want_forced)


def test_sparse_q_full_config3_properties(cuda):
    """Config 3 at TP1: 98,303 keys, 32 Q / 4 KV heads, 4,096 queries (16 gap chunks)."""
    gen = torch.Generator(device=cuda).manual_seed(3)
    ctx = 98304 - 1
    hq, hkv = 32, 4
    key = torch.randn(ctx, hkv, 128, generator=gen, device=cuda).to(torch.bfloat16)
    rng = np.random.default_rng(3)
    chunks = rng.choice(ctx // 256, size=15, replace=False)
    positions = np.sort(np.concatenate([c * 256 + np.arange(256) for c in chunks] +
                                       [np.arange(ctx - 256 + 1, ctx)]))
    queries = torch.randn(positions.size, hq, 128, generator=gen, device=cuda).to(torch.bfloat16)
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    mass = sparse_q_key_mass(queries, key, np.arange(positions.size), positions, 128 ** -0.5,
                             device_error=error)
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    total = float(mass.double().sum())
    rows = positions.size * hq  # every softmax row sums to one
    assert abs(total - rows) <= 1e-3 * rows
    # sampled oracle at full context: 6 queries spread over the prompt
    pick = np.array([0, 255, 1000, 2500, positions.size - 300, positions.size - 1])
    sub = sparse_q_key_mass(queries[pick].contiguous(), key, np.arange(pick.size), positions[pick],
                            128 ** -0.5).cpu().numpy()
    q_np = queries[pick].float().cpu().numpy()
    k_np = key.float().cpu().numpy()
    want = np.zeros(ctx, dtype=np.float64)
    for i, p in enumerate(positions[pick]):
        for h in range(hkv):
            k_h = k_np[: p + 1, h, :]
            for g in range(hq // hkv):
                logits = oracle.round_bf16(q_np[i, h * (hq // hkv) + g] @ k_h.T) * np.float32(128 ** -0.5)
                e = np.exp(logits - logits.max(), dtype=np.float32)
                want[: p + 1] += e / e.sum(dtype=np.float32)
    np.testing.assert_allclose(sub, want, rtol=RTOL, atol=1e-7)


def test_sparse_q_no_queries_and_error_word(cuda):
    key = torch.randn(300, 2, 128, device=cuda).to(torch.bfloat16)
    query = torch.randn(10, 8, 128, device=cuda).to(torch.bfloat16)
    mass = sparse_q_key_mass(query, key, np.zeros(0, dtype=np.int64), np.zeros(0, dtype=np.int64), 0.1)
    assert float(mass.abs().sum()) == 0.0
    with pytest.raises(IndexError):
        sparse_q_key_mass(query, key, np.array([0]), np.array([300]), 0.1)
    with pytest.raises(NotImplementedError):
        sparse_q_key_mass(torch.zeros(4, 8, 64, device=cuda, dtype=torch.bfloat16),
                          torch.zeros(8, 2, 64, device=cuda, dtype=torch.bfloat16), np.array([0]),
                          np.array([1]), 0.1)


def test_sparse_q_abi_bounds_query_rows_and_positions(cuda):
    """Through the C ABI (the Python wrapper would refuse these on the host): a
    query row outside [0, num_query_tokens) or a negative position is not read,
    adds nothing and reports code 4; a position past the last key sees every
    key, as the reference's mask does."""
    import ctypes

    from cacheblend_b200 import _native

    lib = _native.load_library()
    gen = torch.Generator().manual_seed(44)
    key = torch.randn(400, 2, 128, generator=gen).to(torch.bfloat16).to(cuda)
    query = torch.randn(6, 16, 128, generator=gen).to(torch.bfloat16).to(cuda)
    workspace = torch.empty(1 << 22, dtype=torch.uint8, device=cuda)
    aligned = (workspace.data_ptr() + 1023) // 1024 * 1024

    def run(rows, positions):
        rows_d = torch.tensor(rows, dtype=torch.long, device=cuda)
        pos_d = torch.tensor(positions, dtype=torch.long, device=cuda)
        out = torch.empty(400, dtype=torch.float32, device=cuda)
        error = torch.zeros(1, dtype=torch.int32, device=cuda)
        status = lib.cb_sparse_q_scores(
            query.data_ptr(), query.stride(0) * 2, query.shape[0], key.data_ptr(), key.stride(0) * 2, 400,
            16, 2, 128, 0, rows_d.data_ptr(), pos_d.data_ptr(), len(rows), ctypes.c_float(128 ** -0.5),
            out.data_ptr(), aligned, workspace.numel() - (aligned - workspace.data_ptr()), error.data_ptr(),
            _native.stream_handle())
        assert status == 0, lib.cb_last_error().decode()
        torch.cuda.synchronize()
        return out.cpu().numpy(), int(error.item())

    base, err = run([0, 1, 2], [50, 120, 399])
    assert err == 0
    bad_row, err = run([0, 1, 2, 6], [50, 120, 399, 10])  # row 6 does not exist
    assert err == 4
    np.testing.assert_allclose(bad_row, base, rtol=RTOL, atol=1e-6)
    bad_pos, err = run([0, 1, 2, 3], [50, 120, 399, -5])  # negative position
    assert err == 4
    np.testing.assert_allclose(bad_pos, base, rtol=RTOL, atol=1e-6)
    past, err = run([0, 1, 2], [50, 120, 10_000])  # sees every key, like position 399
    assert err == 0
    np.testing.assert_allclose(past, base, rtol=RTOL, atol=1e-6)
