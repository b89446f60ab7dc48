"""The hot-path C-ABI calls can be captured in a CUDA graph: a captured
blend-request step (fused load, deviation, cluster top-k, commit scatter over
every layer; for small rows with the loads on a second stream) replays to
exactly the pages and selection of eager launches."""

from __future__ import annotations

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shard", [1, 8])
def test_graph_replay_matches_eager(cuda, shard):
    """shard 8 (one head per rank) also runs the two-stream pipelined capture."""
    from dataclasses import replace

    shape = replace(bench.CONFIGS[1], layers=6)
    wl = bench.Workload(shape, shard, 0, cuda, host_store=False)
    path = bench.DevicePath(wl)
    stream = torch.cuda.Stream(cuda)
    with torch.cuda.stream(stream):
        path.step(stream)
    torch.cuda.synchronize(cuda)
    pages = [p.clone() for p in wl.pages]
    selected = path.selected.clone()
    scores = path.scores.clone()

    path.capture(stream)
    span = wl.slot_mapping[: wl.plan.allocation_end].to(cuda)
    for p in wl.pages:  # wipe the span: only a replay can restore it
        p[0].view(-1, *p.shape[3:])[span] = 0
        p[1].view(-1, *p.shape[3:])[span] = 0
    path.selected.zero_()
    path.scores.zero_()
    torch.cuda.synchronize(cuda)
    with torch.cuda.stream(stream):
        for _ in range(2):
            path.step(stream)
    torch.cuda.synchronize(cuda)
    path.release()
    assert int(path.device_error.item()) == 0
    for got, want in zip(wl.pages, pages):
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert torch.equal(path.scores, scores)
    assert torch.equal(path.selected, selected)
