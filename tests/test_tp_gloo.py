"""Tensor-parallel host logic on CPU with two gloo ranks: the score all-reduce
used by ``tp_global_selection`` (torch.distributed group and vLLM-style group
coordinator), the rank-identical selection that replaces the reference's
rank-0 broadcast (cacheblend_vllm/ascend.py:764-796), and the reference arm of
bench.py under torchrun (rank 0 prints one line, the other rank exits 0)."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


class _Coordinator:
    """The two attributes of vLLM's GroupCoordinator the selection path uses."""

    def __init__(self, group):
        self.group = group
        self.world_size = dist.get_world_size(group)

    def all_reduce(self, tensor):
        dist.all_reduce(tensor, group=self.group)
        return tensor


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    sys.path[:0] = [str(REPO), str(REPO / "pic-kvcache_b200")]
    import oracle
    from cacheblend_b200.selection import tp_all_reduce, tp_world_size

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(100 + rank)  # each rank's heads give different partial scores
        partial = rng.standard_normal(4096).astype(np.float32)
        gaps = np.random.default_rng(7).random(4096) < 0.2
        total = torch.from_numpy(partial.copy())
        assert tp_world_size(None) == 1 and tp_world_size(dist.group.WORLD) == world
        tp_all_reduce(total, dist.group.WORLD)
        again = tp_all_reduce(torch.from_numpy(partial.copy()), _Coordinator(dist.group.WORLD))
        parts = [None] * world
        dist.all_gather_object(parts, partial)
        expected = np.sum(np.stack(parts), axis=0, dtype=np.float32)
        selected = oracle.select(total.numpy(), gaps, 0.15)
        np.savez(Path(out_dir) / f"rank{rank}.npz", total=total.numpy(), again=again.numpy(),
                 expected=expected, selected=selected)
    finally:
        dist.destroy_process_group()


def test_score_all_reduce_and_identical_selection(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for data in ranks:
        # two-operand float sums are order independent: the reduction is exact
        assert np.array_equal(data["total"], data["expected"])
        assert np.array_equal(data["again"], data["expected"])
    assert np.array_equal(ranks[0]["selected"], ranks[1]["selected"])
    assert ranks[0]["selected"].size > 0


def test_bench_reference_arm_under_torchrun():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(REPO / "bench.py"),
           "--impl", "reference", "--gpus", "2", "--config", "1", "--steps", "1", "--warmup", "0"]
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [line for line in proc.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
    # the same workload description as the GPU arm prints
    assert line["config"]["workload"] == "qwen3-0.6b-cpu-plumbing" and line["config"]["parallelism"] == "tp2"


def _peer_rank_main(rank: int, world: int, port: int, out_dir: str, fail_open_rank: int = -1) -> None:
    """PeerScoreExchange's host protocol over two gloo ranks with the C ABI faked:
    IPC handles swapped through the group, the address table in rank order (own
    buffer at this rank, the others' mappings elsewhere), the select's arguments,
    and the teardown order (unmap every peer, then free the own buffer)."""
    import ctypes

    sys.path[:0] = [str(REPO), str(REPO / "pic-kvcache_b200")]
    from cacheblend_b200 import peer_exchange

    calls, seen = [], {}

    def fake_call(name, *args):
        calls.append(name)
        if name == "cb_peer_select_buffer_size":
            ctypes.c_int64.from_address(args[2]).value = 4096
        elif name == "cb_peer_buffer_create":
            ctypes.c_uint64.from_address(args[2]).value = 0x10000 * (rank + 1)
            (ctypes.c_uint8 * 64).from_address(args[3])[0] = rank + 1  # the "handle" names its owner
        elif name == "cb_peer_buffer_open":
            if rank == fail_open_rank:
                raise RuntimeError("cb_peer_buffer_open: peer access unsupported")
            owner = (ctypes.c_uint8 * 64).from_address(args[1])[0] - 1
            ctypes.c_uint64.from_address(args[2]).value = 0x1000000 * (owner + 1) + 0x100 * (rank + 1)
        elif name == "cb_select_topk_peer":
            _, _, n, k, _, cap, table, r, w, max_tokens, protocol = args[:11]
            seen.update(n=n, k=k, cap=cap, rank=r, world=w, max_tokens=max_tokens, protocol=protocol,
                        table=list((ctypes.c_uint64 * w).from_address(table)))
        elif name in ("cb_peer_buffer_close", "cb_peer_buffer_destroy"):
            calls[-1] = f"{name}:{args[1]:#x}"

    peer_exchange._native.call = fake_call
    peer_exchange._native.require_cuda = lambda *tensors: None
    peer_exchange._native.stream_handle = lambda stream=None: 0
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        try:
            exchange = peer_exchange.PeerScoreExchange(dist.group.WORLD, 1000, "cpu")
        except peer_exchange.PeerExchangeUnavailable as error:
            (Path(out_dir) / f"peer{rank}.json").write_text(json.dumps({"calls": calls, "error": str(error)}))
            return
        selected = exchange.select(torch.zeros(1000), torch.zeros(1000, dtype=torch.uint8), 150, 170)
        exchange.close()
        exchange.close()  # idempotent
        (Path(out_dir) / f"peer{rank}.json").write_text(json.dumps(
            {"calls": calls, "seen": seen, "selected": int(selected.numel())}))
    finally:
        dist.destroy_process_group()


def test_peer_exchange_host_protocol(tmp_path):
    world = 2
    mp.start_processes(_peer_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for rank in range(world):
        got = json.loads((tmp_path / f"peer{rank}.json").read_text())
        other = 1 - rank
        mapped = 0x1000000 * (other + 1) + 0x100 * (rank + 1)
        table = [0, 0]
        table[rank] = 0x10000 * (rank + 1)
        table[other] = mapped
        assert got["seen"] == {"n": 1000, "k": 150, "cap": 170, "rank": rank, "world": world,
                               "max_tokens": 1000, "protocol": 0, "table": table}
        assert got["selected"] == 170
        assert got["calls"] == ["cb_peer_select_buffer_size", "cb_peer_buffer_create", "cb_peer_buffer_open",
                                "cb_select_topk_peer", f"cb_peer_buffer_close:{mapped:#x}",
                                f"cb_peer_buffer_destroy:{0x10000 * (rank + 1):#x}"]


def test_peer_exchange_setup_failure_is_collective(tmp_path):
    """A rank that cannot map a peer's buffer: every rank raises PeerExchangeUnavailable
    (callers then fall back to the NCCL all-reduce together), mappings are closed before
    any owner frees its buffer, and nothing is left allocated."""
    world = 2
    mp.start_processes(_peer_rank_main, args=(world, _free_port(), str(tmp_path), 1), nprocs=world,
                       start_method="spawn", join=True)
    rank0 = json.loads((tmp_path / "peer0.json").read_text())
    rank1 = json.loads((tmp_path / "peer1.json").read_text())
    for got in (rank0, rank1):
        assert "rank 1 mapping rank 0" in got["error"]
    mapped = 0x1000000 * 2 + 0x100 * 1  # rank 0's mapping of rank 1's buffer
    assert rank0["calls"] == ["cb_peer_select_buffer_size", "cb_peer_buffer_create", "cb_peer_buffer_open",
                              f"cb_peer_buffer_close:{mapped:#x}", f"cb_peer_buffer_destroy:{0x10000:#x}"]
    assert rank1["calls"] == ["cb_peer_select_buffer_size", "cb_peer_buffer_create", "cb_peer_buffer_open",
                              f"cb_peer_buffer_destroy:{0x20000:#x}"]
