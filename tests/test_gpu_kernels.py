"""GPU parity of the hot-path kernels against the CPU oracle and the golden
vectors of the reference: bit-exact KV bytes and index sets; deviation scores
bit-exact against the oracle (same association order) and within 1e-5 of the
reference's torch sum.  All calls go through the product API / C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.config import CacheBlendConfig
from cacheblend_b200.kv_layout import describe_paged, gather_chunk_major, gather_paged_kv, scatter_paged_kv
from cacheblend_b200.loader import PagedBlendLoader
from cacheblend_b200.rope import relocate_key
from cacheblend_b200.selection import kv_deviation, recompute_budget, select_from_scores, select_tokens
from cacheblend_b200.storage import LocalPinnedCPUStore
from cacheblend_b200.types import BlendPlan, BlendSegment

pytestmark = pytest.mark.gpu


def bf16(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


# ------------------------------------------------------------------ K1 gather/scatter
@pytest.mark.parametrize("layout", ["merged_first", "merged_block", "separate"])
def test_gather_scatter_golden(golden, cuda, layout):
    base = bf16(golden["kv_base"], cuda)
    if layout == "merged_first":
        paged = base.clone()
    elif layout == "merged_block":
        paged = base.permute(1, 0, 2, 3, 4).contiguous()
    else:
        paged = [base[0].clone(), base[1].clone()]
    slots = torch.from_numpy(golden["kv_slots"])
    assert np.array_equal(bits(gather_paged_kv(paged, slots, 4)), golden[f"kv_gather_{layout}"])
    scatter_paged_kv(bf16(golden["kv_replacement"], cuda)[:, :5], paged, slots[:5], 4)
    after = paged if isinstance(paged, torch.Tensor) else torch.stack(paged)
    if layout == "merged_block":
        after = after.permute(1, 0, 2, 3, 4)
    assert np.array_equal(bits(after), golden[f"kv_scatter_{layout}"])


@pytest.mark.parametrize("layout", ["merged_first", "merged_block", "separate"])
def test_reference_known_answer_float32(cuda, layout):
    # reference tests/test_kv_layout.py:7-40 (8-byte rows: non-16B vector path)
    base = torch.arange(2 * 3 * 2 * 2, dtype=torch.float32, device=cuda).reshape(2, 3, 2, 2)
    if layout == "merged_first":
        paged = base.clone()
    elif layout == "merged_block":
        paged = base.permute(1, 0, 2, 3).contiguous()
    else:
        paged = [base[0].clone(), base[1].clone()]
    slots = torch.tensor([0, 3, 4])
    gathered = gather_paged_kv(paged, slots, 2)
    assert torch.equal(gathered, base[:, [0, 1, 2], [0, 1, 0]])
    replacement = torch.full_like(gathered, -1)
    scatter_paged_kv(replacement, paged, slots, 2)
    assert torch.equal(gather_paged_kv(paged, slots, 2), replacement)
    out = torch.empty(2, 3, 2, device=cuda)
    assert gather_paged_kv(paged, slots, 2, out=out) is out


def test_rejects_unknown_layout_and_cpu_tensors(cuda):
    with pytest.raises(ValueError, match="unsupported"):
        gather_paged_kv(torch.empty(3, 4, 5, device=cuda), torch.tensor([0]), 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        gather_paged_kv(torch.zeros(2, 3, 2, 2), torch.tensor([0]), 2)
    with pytest.raises(IndexError):
        gather_paged_kv(torch.zeros(2, 3, 2, 2, device=cuda), torch.tensor([6]), 2)


@pytest.mark.parametrize("hnd", [False, True])
def test_gather_scatter_qwen3_8b_layer_bit_exact(cuda, hnd):
    gen = torch.Generator(device=cuda).manual_seed(3)
    nb, bs, h, d, tokens = 2304, 16, 8, 128, 4096
    if hnd:  # [2, NB, H, BS, D] storage seen as [2, NB, BS, H, D]
        cache = torch.randn(2, nb, h, bs, d, generator=gen, device=cuda).to(torch.bfloat16).transpose(2, 3)
    else:
        cache = torch.randn(2, nb, bs, h, d, generator=gen, device=cuda).to(torch.bfloat16)
    slots = torch.randperm(nb * bs)[:tokens]
    got = gather_paged_kv(cache, slots, bs)
    k_np = bits(cache[0])
    v_np = bits(cache[1])
    assert np.array_equal(bits(got), oracle.paged_gather(k_np, v_np, slots.numpy(), bs))
    new = torch.randn(2, tokens, h, d, generator=gen, device=cuda).to(torch.bfloat16)
    scatter_paged_kv(new, cache, slots, bs)
    oracle.paged_scatter(bits(new), k_np, v_np, slots.numpy(), bs)
    assert np.array_equal(bits(cache[0]), k_np) and np.array_equal(bits(cache[1]), v_np)


def test_chunk_major_store_staging(cuda):
    gen = torch.Generator(device=cuda).manual_seed(4)
    cache = torch.randn(2, 64, 16, 4, 128, generator=gen, device=cuda).to(torch.bfloat16)
    paged = describe_paged(cache, 16)
    slots = torch.randperm(64 * 16)[:512].to(cuda)
    staging = torch.empty(2, 2, 256, 4, 128, dtype=torch.bfloat16, device=cuda)  # [chunks, K/V, C, H, D]
    gather_chunk_major(paged, slots, staging)
    want = gather_paged_kv(cache, slots, 16)  # [2, 512, H, D]
    for c in range(2):
        assert torch.equal(staging[c], want[:, c * 256 : (c + 1) * 256])


# ------------------------------------------------------------------ K2 relocation + load
class _Rope:
    def __init__(self, cos_sin: np.ndarray, head_size: int, neox: bool, device):
        self.head_size = head_size
        self.rotary_dim = cos_sin.shape[1]
        self.is_neox_style = neox
        self.cos_sin_cache = torch.from_numpy(cos_sin).to(device)


@pytest.mark.parametrize("name", ["bf16_neox", "bf16_gptj", "fp32_neox", "bf16_partial"])
def test_relocate_key_golden(golden, cuda, name):
    rope = _Rope(golden[f"rope_{name}_cos_sin"], 64, "gptj" not in name, cuda)
    key_bits = golden[f"rope_{name}_key"]
    key = torch.from_numpy(key_bits).to(cuda) if name.startswith("fp32") else bf16(key_bits, cuda)
    out = relocate_key(rope, torch.from_numpy(golden[f"rope_{name}_old"]),
                       torch.from_numpy(golden[f"rope_{name}_new"]), key)
    assert np.array_equal(bits(out), golden[f"rope_{name}_out"])


def _golden_loader_inputs(golden, tag, device, pinned: bool):
    apc, alloc_end, bs, chunk, layers = (int(x) for x in golden[f"loader_{tag}_meta"])
    plan_rows = golden[f"loader_{tag}_plan"]
    store = LocalPinnedCPUStore(chunk, 1 << 26, pin_memory=pinned)
    segments = []
    for i, (src, tgt, n) in enumerate(plan_rows):
        sid = store.begin_put("m", int(src), list(range(1000 * (i + 1), 1000 * (i + 1) + chunk)), layers)
        for layer in range(layers):
            host_bits = golden[f"loader_{tag}_host_{i}_{layer}"]
            parent = torch.zeros(2, 3 * chunk, *host_bits.shape[2:], dtype=torch.bfloat16)
            if pinned:
                parent = parent.pin_memory()
            parent[:, chunk : 2 * chunk] = torch.from_numpy(host_bits.view(np.int16)).view(torch.bfloat16)
            store.put_layer_host(sid, layer, parent[:, chunk : 2 * chunk])  # non-contiguous view
        segments.append(BlendSegment(sid, int(tgt)))
    store.pin("r", segments)
    plan = BlendPlan.from_segments(apc, segments)
    pages = [bf16(golden[f"loader_{tag}_pages_before"][layer], device) for layer in range(layers)]
    config = CacheBlendConfig.from_extra_config(
        {"chunk_size": chunk, "local_cpu_gb": 0.01, "strict_version_check": False,
         "fused_segment_copy": tag == "fused"}
    )
    rope = _Rope(golden[f"loader_{tag}_cos_sin"], golden[f"loader_{tag}_cos_sin"].shape[1], True, device)
    slot_mapping = torch.from_numpy(golden[f"loader_{tag}_slot_mapping"])
    return store, plan, pages, config, rope, slot_mapping, bs, layers, apc


@pytest.mark.parametrize("mode", ["copy", "zerocopy"])
@pytest.mark.parametrize("tag", ["fused", "individual"])
def test_loader_golden(golden, cuda, monkeypatch, tag, mode):
    monkeypatch.setenv("CACHEBLEND_B200_LOAD", mode)
    store, plan, pages, config, rope, slot_mapping, bs, layers, apc = _golden_loader_inputs(
        golden, tag, cuda, pinned=True
    )
    loader = PagedBlendLoader(pages, store, "r", plan, slot_mapping, bs, config,
                              load_stream=torch.cuda.Stream(cuda))
    loader.prefetch(0, rope)
    for layer in range(layers):
        staging = loader.get(layer)
        loader.prefetch(layer + 1, rope)
        assert np.array_equal(bits(staging), golden[f"loader_{tag}_staging_{layer}"]), layer
        recomputed = bf16(golden[f"loader_{tag}_recomputed_{layer}"], cuda)
        staging.copy_(recomputed)
        loader.commit(layer, staging)
        assert np.array_equal(bits(pages[layer]), golden[f"loader_{tag}_pages_after_{layer}"]), layer


def test_loader_without_event_pipeline_and_pageable_store(golden, cuda):
    store, plan, pages, config, rope, slot_mapping, bs, layers, apc = _golden_loader_inputs(
        golden, "fused", cuda, pinned=False
    )
    config = CacheBlendConfig.from_extra_config(
        {"chunk_size": 8, "local_cpu_gb": 0.01, "strict_version_check": False, "event_pipeline": False}
    )
    loader = PagedBlendLoader(pages, store, "r", plan, slot_mapping, bs, config)
    loader.prefetch(0, rope)
    assert np.array_equal(bits(loader.get(0)), golden["loader_fused_staging_0"])


def _random_blend_case(seed, device, heads=8, hd=128, tokens=4096, chunk=256, hits=12, bs=16, pool=2048,
                       apc=0, max_pos=40960):
    rng = np.random.default_rng(seed)
    chunks = tokens // chunk
    hit_idx = np.sort(rng.choice(np.arange(apc // chunk, chunks), size=hits, replace=False))
    sources = rng.integers(0, max_pos - chunk, size=hits)
    k = (rng.integers(0, 1 << 16, size=(pool, bs, heads, hd), dtype=np.uint16) & 0xBFFF)
    v = (rng.integers(0, 1 << 16, size=(pool, bs, heads, hd), dtype=np.uint16) & 0xBFFF)
    blocks = rng.permutation(pool)[: tokens // bs]
    slots = (blocks[:, None] * bs + np.arange(bs)[None, :]).reshape(-1).astype(np.int64)
    hosts = [rng.integers(0, 1 << 16, size=(2, chunk, heads, hd), dtype=np.uint16) & 0xBFFF for _ in range(hits)]
    inv = 1.0 / (1e6 ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    freqs = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    cos_sin = np.concatenate((np.cos(freqs), np.sin(freqs)), axis=-1).astype(np.float32)
    return hit_idx, sources, k, v, slots, hosts, cos_sin


@pytest.mark.parametrize("apc", [0, 512])
def test_blend_load_cfg1_shapes_vs_oracle(cuda, apc):
    """Config-1 shapes (Qwen3-0.6B KV: 8 heads x 128, 4096 tokens, 12/16 hits)."""
    chunk, bs = 256, 16
    hit_idx, sources, k, v, slots, hosts, cos_sin = _random_blend_case(5 + apc, cuda, apc=apc)
    store = LocalPinnedCPUStore(chunk, 1 << 30)
    segments = []
    for i, c in enumerate(hit_idx):
        sid = store.begin_put("m", int(sources[i]), list(range(i * chunk, (i + 1) * chunk)), 1)
        store.put_layer_host(sid, 0, torch.from_numpy(hosts[i].view(np.int16)).view(torch.bfloat16).pin_memory())
        segments.append(BlendSegment(sid, int(c) * chunk))
    store.pin("r", segments)
    plan = BlendPlan.from_segments(apc, segments)
    pages = [torch.stack([bf16(k, cuda), bf16(v, cuda)])]
    config = CacheBlendConfig.from_extra_config({"chunk_size": chunk, "strict_version_check": False})
    rope = _Rope(cos_sin, 128, True, cuda)
    loader = PagedBlendLoader(pages, store, "r", plan, torch.from_numpy(slots), bs, config,
                              load_stream=torch.cuda.Stream(cuda))
    loader.prefetch(0, rope)
    got = bits(loader.get(0))
    table = oracle.f32_to_bf16(cos_sin)
    segs = [(int(sources[i]), int(c) * chunk, chunk, hosts[i]) for i, c in enumerate(hit_idx)]
    want = oracle.blend_load(oracle.BF16, plan.allocation_end, apc, k, v, slots[: plan.allocation_end], bs,
                             segs, np.ones(len(segs), dtype=np.int32), table, 128, 128, True)
    assert np.array_equal(got, want)


# ------------------------------------------------------------------ K3 deviation + select
def test_deviation_golden_and_oracle(golden, cuda):
    fresh = bf16(golden["dev_fresh"], cuda)
    cached = bf16(golden["dev_cached"], cuda)
    scores = kv_deviation(fresh, cached, torch.from_numpy(golden["dev_absolute"]))
    np.testing.assert_allclose(scores.cpu().numpy(), golden["dev_scores"], rtol=1e-5)
    want = oracle.kv_deviation(golden["dev_fresh"], golden["dev_cached"], oracle.BF16,
                               abs_index=golden["dev_absolute"])
    assert np.array_equal(scores.cpu().numpy(), want)


@pytest.mark.parametrize("width,dtype", [(1024, torch.bfloat16), (512, torch.float16), (256, torch.float32),
                                         (100, torch.bfloat16),
                                         # rows of <= 32 16-byte units: tokens packed per warp
                                         (256, torch.bfloat16), (128, torch.bfloat16), (64, torch.float16),
                                         (32, torch.float32), (8, torch.bfloat16)])
def test_deviation_bit_exact_vs_oracle(cuda, width, dtype):
    gen = torch.Generator(device=cuda).manual_seed(width)
    n, total = 3000, 4000
    cached = torch.randn(total, width, generator=gen, device=cuda).to(dtype)
    fresh = (cached[500 : 500 + n].float() + 0.05 * torch.randn(n, width, generator=gen, device=cuda)).to(dtype)
    scores = kv_deviation(fresh, cached, absolute_offset=500)
    code = {torch.bfloat16: oracle.BF16, torch.float16: oracle.FP16, torch.float32: oracle.FP32}[dtype]
    want = oracle.kv_deviation(bits(fresh), bits(cached), code, abs_offset=500)
    assert np.array_equal(scores.cpu().numpy(), want)
    ref = ((fresh.float() - cached[500 : 500 + n].float()) ** 2).sum(-1)
    torch.testing.assert_close(scores, ref, rtol=1e-5, atol=0)


@pytest.mark.parametrize("width", [128, 1024])
def test_deviation_out_of_range_rows_are_nan(cuda, width):
    gen = torch.Generator(device=cuda).manual_seed(7)
    cached = torch.randn(100, width, generator=gen, device=cuda).to(torch.bfloat16)
    fresh = torch.randn(37, width, generator=gen, device=cuda).to(torch.bfloat16)
    index = torch.arange(37, dtype=torch.int64) * 2  # in range except the three set below
    index[[0, 5, 36]] = torch.tensor([-1, 100, 500])
    scores = kv_deviation(fresh, cached, index).cpu().numpy()
    want = oracle.kv_deviation(bits(fresh), bits(cached), oracle.BF16, abs_index=index.numpy().clip(0, 99))
    bad = np.zeros(37, dtype=bool)
    bad[[0, 5, 36]] = True
    assert np.isnan(scores[bad]).all()
    assert np.array_equal(scores[~bad], want[~bad])


@pytest.mark.parametrize("case", range(6))
def test_select_golden(golden, cuda, case):
    forced = golden[f"sel_{case}_forced"] if golden[f"sel_{case}_has_forced"][0] else None
    scores = torch.from_numpy(golden[f"sel_{case}_scores"]).to(cuda)
    out = select_tokens(scores, golden[f"sel_{case}_gaps"], float(golden[f"sel_{case}_ratio"][0]), forced)
    assert np.array_equal(out.cpu().numpy(), golden[f"sel_{case}_out"])


@pytest.mark.parametrize("n", [1, 2, 7, 31, 1024, 1025, 32768, 65535, 98303, 344_064, 344_065, 400_000])
def test_select_vs_oracle_random_with_ties(cuda, n):
    rng = np.random.default_rng(n)
    scores = rng.integers(0, max(4, n // 8), size=n).astype(np.float32)  # many ties
    gaps = rng.random(n) < 0.25
    forced = rng.random(n) < 0.05
    for ratio in (0.0, 0.15, 0.5, 1.0):
        got = select_tokens(torch.from_numpy(scores).to(cuda), gaps, ratio, forced).cpu().numpy()
        assert np.array_equal(got, oracle.select(scores, gaps, ratio, forced)), ratio


def test_select_special_values(cuda):
    scores = np.array([np.nan, 1.0, -0.0, 0.0, np.inf, -np.inf, 3.0, np.nan], dtype=np.float32)
    gaps = np.zeros(8, dtype=bool)
    got = select_tokens(torch.from_numpy(scores).to(cuda), gaps, 0.5).cpu().numpy()
    assert np.array_equal(got, oracle.select(scores, gaps, 0.5))
    assert got.tolist() == [0, 4, 6, 7]


@pytest.mark.parametrize("n", [100, 20_000, 300_000])
def test_select_all_base_and_empty_budget(cuda, n):
    """k = 0 (every token a gap): the base set alone, also when each cluster CTA
    holds more keys than it has threads (its compaction then reads entries
    other threads loaded)."""
    scores = torch.rand(n, device=cuda)
    base = torch.ones(n, dtype=torch.uint8, device=cuda)
    assert np.array_equal(select_from_scores(scores, base, 0, n).cpu().numpy(), np.arange(n))
    assert recompute_budget(n, n, n, 0.5) == 0


def test_select_reference_known_answers(cuda):
    # reference tests/test_ascend.py:144-154, 256-267
    out = select_tokens(torch.tensor([1.0, 10.0, 2.0, 9.0], device=cuda), np.array([1, 0, 1, 0], bool), 0.5)
    assert out.cpu().tolist() == [0, 1, 2]
    out = select_tokens(torch.tensor([0.0, 1.0, 10.0, 9.0], device=cuda), np.array([1, 0, 0, 0], bool), 0.5,
                        forced_mask=np.array([0, 1, 0, 0], bool))
    assert out.cpu().tolist() == [0, 1, 2]


def test_deviation_select_full_cfg4_size(cuda):
    """Config 4 size (65,535 active tokens, 8 heads): scores and index set vs oracle."""
    gen = torch.Generator(device=cuda).manual_seed(44)
    n, width = 65535, 1024
    cached = torch.randn(n + 1, width, generator=gen, device=cuda).to(torch.bfloat16)
    fresh = (cached[1:].float() + 0.05 * torch.randn(n, width, generator=gen, device=cuda)).to(torch.bfloat16)
    scores = kv_deviation(fresh, cached, absolute_offset=1)
    want = oracle.kv_deviation(bits(fresh), bits(cached), oracle.BF16, abs_offset=1)
    assert np.array_equal(scores.cpu().numpy(), want)
    gaps = np.zeros(n, dtype=bool)
    gaps[np.random.default_rng(1).choice(n // 256, 64, replace=False)[:, None] * 256 + np.arange(256)] = True
    got = select_tokens(scores, gaps, 0.15).cpu().numpy()
    assert np.array_equal(got, oracle.select(want, gaps, 0.15))
    assert np.all(np.diff(got) > 0)


@pytest.mark.parametrize("na,nb", [(0, 5), (5, 0), (1, 1), (1000, 3000), (70000, 90000)])
def test_selection_overlap_vs_numpy(cuda, na, nb):
    from cacheblend_b200.selection import selection_overlap

    rng = np.random.default_rng(na + nb)
    universe = max(na, nb) * 2 + 1
    a = np.sort(rng.choice(universe, size=na, replace=False))
    b = np.sort(rng.choice(universe, size=nb, replace=False))
    overlap, union = selection_overlap(torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda))
    assert overlap == len(np.intersect1d(a, b)) and union == len(np.union1d(a, b))
