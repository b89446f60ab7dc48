"""The TP selection with the score reduction over peer memory
(cb_select_topk_peer): the all-reduce and ``_select`` of
cacheblend_vllm/ascend.py:764-796 in one kernel per rank.  Every rank's sum
must equal the rank-order fp32 sum of the partial scores bit for bit, and
every rank's index set the oracle's select over that sum exactly.

On one GPU the protocol runs with every rank played by one cooperative launch
(cluster r = rank r): ranks 1, 2, 4 and 8, several calls in a row (the call
counters and the two receive buffers alternate), NaN partials, ties, every
token a gap, no token at all, token counts that are not multiples of 4.  With
two or more GPUs the real exchange runs between processes, one per GPU,
mapping each other's buffers through CUDA IPC, eagerly and from a CUDA graph."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.peer_exchange import AllRanksExchange
from cacheblend_b200.selection import recompute_budget

pytestmark = pytest.mark.gpu


def rank_order_sum(partials: np.ndarray) -> np.ndarray:
    total = partials[0].astype(np.float32)
    for row in partials[1:]:
        total = (total + row.astype(np.float32)).astype(np.float32)
    return total


def _partials(world: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    # per-rank deviation shares: non-negative, a few orders of magnitude apart
    return (rng.random((world, n)) ** 3 * 10.0 ** rng.integers(-2, 3, (world, n))).astype(np.float32)


def _check(exchange, partials: np.ndarray, gaps: np.ndarray, ratio: float, device) -> None:
    world, n = partials.shape
    k = recompute_budget(n, int(gaps.sum()), int(gaps.sum()), ratio)
    cap = int(gaps.sum()) + k
    base = torch.from_numpy(gaps.astype(np.uint8)).to(device)
    selected, summed = exchange.select(torch.from_numpy(partials).to(device), base, k, cap)
    torch.cuda.synchronize(device)
    assert int(exchange.device_error.item()) == 0
    want_sum = rank_order_sum(partials)
    want = oracle.select(want_sum, gaps, ratio)
    got_sum = summed.cpu().numpy()
    got = selected.cpu().numpy()
    for r in range(world):
        assert np.array_equal(got_sum[r], want_sum, equal_nan=True), r
        assert np.array_equal(got[r], want), r


PROTOCOLS = ["flags", "low_latency"]


@pytest.mark.parametrize("protocol", PROTOCOLS)
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_all_ranks_match_oracle_call_after_call(cuda, world, protocol):
    n = 32768
    exchange = AllRanksExchange(world, n, cuda, protocol)
    for call in range(5):  # both receive buffers twice, counters 1..5
        partials = _partials(world, n, 100 * world + call)
        gaps = np.random.default_rng(call).random(n) < 0.1
        _check(exchange, partials, gaps, 0.15, cuda)


@pytest.mark.parametrize("protocol", PROTOCOLS)
@pytest.mark.parametrize("n", [1, 5, 7, 1001, 40_003])
def test_all_ranks_ragged_sizes(cuda, n, protocol):
    exchange = AllRanksExchange(4, 40_003, cuda, protocol)
    for call in range(2):
        partials = _partials(4, n, n + call)
        gaps = np.zeros(n, dtype=bool)
        gaps[::9] = True
        _check(exchange, partials, gaps, 0.2, cuda)


@pytest.mark.parametrize("protocol", PROTOCOLS)
def test_all_ranks_nan_ties_and_edge_masks(cuda, protocol):
    n, world = 20_000, 4
    exchange = AllRanksExchange(world, n, cuda, protocol)
    partials = np.ones((world, n), dtype=np.float32)
    partials[:, ::5] = 2.0          # exact ties at the threshold
    partials[1, [7, 300, 19_999]] = np.nan  # out-of-range cached rows on one rank rank first
    gaps = np.zeros(n, dtype=bool)
    gaps[1000:1100] = True
    _check(exchange, partials, gaps, 0.1, cuda)
    _check(exchange, _partials(world, n, 3), np.ones(n, dtype=bool), 0.1, cuda)   # k = 0
    _check(exchange, _partials(world, n, 4), np.zeros(n, dtype=bool), 0.1, cuda)  # no gap
    # no token at all: the call still exchanges (the counters stay in step)
    empty = torch.empty(world, 0, dtype=torch.float32, device=cuda)
    sel, _ = exchange.select(empty, torch.empty(0, dtype=torch.uint8, device=cuda), 0, 0)
    torch.cuda.synchronize(cuda)
    assert sel.numel() == 0 and int(exchange.device_error.item()) == 0
    _check(exchange, _partials(world, n, 5), gaps, 0.1, cuda)


def test_abi_rejects_bad_arguments(cuda):
    from cacheblend_b200 import _native
    import ctypes

    lib = _native.load_library()
    size = ctypes.c_int64(0)
    assert lib.cb_peer_select_buffer_size(9, 100, ctypes.byref(size)) == _native.CB_ERR_INVALID
    assert lib.cb_peer_select_buffer_size(2, 8 * 42 * 1024 + 1, ctypes.byref(size)) == _native.CB_ERR_INVALID
    assert lib.cb_peer_select_buffer_size(2, 100, ctypes.byref(size)) == 0 and size.value > 0
    scores = torch.zeros(100, device=cuda)
    base = torch.zeros(100, dtype=torch.uint8, device=cuda)
    out = torch.empty(100, dtype=torch.long, device=cuda)
    buffers = (ctypes.c_uint64 * 2)(0, 0)  # null exchange buffers
    rc = lib.cb_select_topk_peer(ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(base.data_ptr()), 100, 5,
                                 ctypes.c_void_p(out.data_ptr()), 100, buffers, 0, 2, 100, 0, None, None, None)
    assert rc == _native.CB_ERR_INVALID
    real = [torch.zeros(size.value, dtype=torch.uint8, device=cuda) for _ in range(2)]
    buffers = (ctypes.c_uint64 * 2)(*[b.data_ptr() for b in real])
    rc = lib.cb_select_topk_peer(ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(base.data_ptr()), 200, 5,
                                 ctypes.c_void_p(out.data_ptr()), 100, buffers, 0, 2, 100, 0, None, None, None)
    assert rc == _native.CB_ERR_INVALID  # more tokens than the exchange was sized for
    rc = lib.cb_select_topk_peer(ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(base.data_ptr()), 100, 5,
                                 ctypes.c_void_p(out.data_ptr()), 100, buffers, 2, 2, 100, 0, None, None, None)
    assert rc == _native.CB_ERR_INVALID  # rank outside the world
    rc = lib.cb_select_topk_peer(ctypes.c_void_p(scores.data_ptr()), ctypes.c_void_p(base.data_ptr()), 100, 5,
                                 ctypes.c_void_p(out.data_ptr()), 100, buffers, 0, 2, 100, 2, None, None, None)
    assert rc == _native.CB_ERR_INVALID  # no such protocol


# ---- real ranks: one process per GPU ------------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str, protocol: str = "flags") -> None:
    import torch.distributed as dist

    from cacheblend_b200.peer_exchange import PeerScoreExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    n = 32768
    exchange = PeerScoreExchange(dist.group.WORLD, n, device, protocol)
    results = {}
    try:
        gaps = np.random.default_rng(7).random(n) < 0.1
        base = torch.from_numpy(gaps.astype(np.uint8)).to(device)
        k = recompute_budget(n, int(gaps.sum()), int(gaps.sum()), 0.15)
        cap = int(gaps.sum()) + k
        summed = torch.empty(n, dtype=torch.float32, device=device)
        for call in range(4):
            partial = torch.from_numpy(_partials(world, n, 50 + call)[rank]).to(device)
            sel = exchange.select(partial, base, k, cap, summed=summed)
            results[f"eager{call}"] = sel.cpu().numpy()
            results[f"sum{call}"] = summed.cpu().numpy()
        # the same exchange replayed from a CUDA graph, three times
        stream = torch.cuda.Stream(device)
        partial = torch.from_numpy(_partials(world, n, 90)[rank]).to(device)
        torch.cuda.synchronize(device)
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            captured = exchange.select(partial, base, k, cap, stream=stream)
        dist.barrier()
        for rep in range(3):
            graph.replay()
            torch.cuda.synchronize(device)
            results[f"graph{rep}"] = captured.cpu().numpy()
        del graph
        results["error"] = np.array([int(exchange.device_error.item())])
    finally:
        exchange.close()
        dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **results)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two or more GPUs")
@pytest.mark.parametrize("protocol", PROTOCOLS)
def test_processes_exchange_over_nvlink(tmp_path, protocol):
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    world = 1 << (world.bit_length() - 1)  # 2, 4 or 8
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), protocol), nprocs=world,
                       start_method="spawn")
    got = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    n = 32768
    gaps = np.random.default_rng(7).random(n) < 0.1
    for call in range(4):
        want_sum = rank_order_sum(_partials(world, n, 50 + call))
        want = oracle.select(want_sum, gaps, 0.15)
        for r in range(world):
            assert np.array_equal(got[r][f"sum{call}"], want_sum), (call, r)
            assert np.array_equal(got[r][f"eager{call}"], want), (call, r)
    want = oracle.select(rank_order_sum(_partials(world, n, 90)), gaps, 0.15)
    for r in range(world):
        assert int(got[r]["error"][0]) == 0
        for rep in range(3):
            assert np.array_equal(got[r][f"graph{rep}"], want), (rep, r)
