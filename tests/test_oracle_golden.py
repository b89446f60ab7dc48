"""Pin the CPU oracle to the reference: golden vectors produced by the
reference implementation (tests/golden/make_golden.py) and the reference's
own known-answer tests (tests/test_kv_layout.py, tests/test_ascend.py of the
reference), re-checked here against ``oracle``.  CPU only."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from oracle import BF16, FP32


@pytest.mark.parametrize("layout", ["merged_first", "merged_block", "separate"])
def test_paged_gather_scatter_match_reference(golden, layout):
    base = golden["kv_base"]
    slots = golden["kv_slots"]
    k, v = (np.ascontiguousarray(p) for p in (base[0], base[1]))
    gathered = oracle.paged_gather(k, v, slots, 4)
    assert np.array_equal(gathered, golden[f"kv_gather_{layout}"])
    oracle.paged_scatter(golden["kv_replacement"][:, :5], k, v, slots[:5], 4)
    assert np.array_equal(np.stack([k, v]), golden[f"kv_scatter_{layout}"])


def test_reference_known_answer_gather_round_trip():
    # reference tests/test_kv_layout.py:7-24: slots [0, 3, 4], block_size 2
    base = np.arange(2 * 3 * 2 * 2, dtype=np.float32).reshape(2, 3, 2, 2)
    k, v = base[0].copy(), base[1].copy()
    slots = np.array([0, 3, 4])
    gathered = oracle.paged_gather(k, v, slots, 2)
    assert np.array_equal(gathered, base[:, [0, 1, 2], [0, 1, 0]])
    replacement = np.full_like(gathered, -1)
    oracle.paged_scatter(replacement, k, v, slots, 2)
    assert np.array_equal(oracle.paged_gather(k, v, slots, 2), replacement)


def test_gather_rejects_out_of_range_slot():
    k = np.zeros((3, 2, 4), dtype=np.float32)
    with pytest.raises(IndexError):
        oracle.paged_gather(k, k.copy(), np.array([6]), 2)


@pytest.mark.parametrize("name", ["bf16_neox", "bf16_gptj", "fp32_neox", "bf16_partial"])
def test_relocate_matches_reference_bit_exact(golden, name):
    dtype = FP32 if name.startswith("fp32") else BF16
    cos_sin = golden[f"rope_{name}_cos_sin"]
    rotary_dim = cos_sin.shape[1]
    table = cos_sin if dtype == FP32 else oracle.f32_to_bf16(cos_sin)
    out = oracle.relocate(
        golden[f"rope_{name}_key"], table, golden[f"rope_{name}_old"], golden[f"rope_{name}_new"],
        64, rotary_dim, "gptj" not in name, dtype,
    )
    assert np.array_equal(out, golden[f"rope_{name}_out"])


def test_relocate_identity_positions_still_round(golden):
    # torch.equal(old, new) is False overall, so rows whose own positions are
    # equal still go through the bf16 delta rotation (ascend.py:64-65)
    name = "bf16_neox"
    key = golden[f"rope_{name}_key"]
    out = golden[f"rope_{name}_out"]
    assert np.array_equal(golden[f"rope_{name}_old"][:3], golden[f"rope_{name}_new"][:3])
    assert out.shape == key.shape


@pytest.mark.parametrize("tag", ["fused", "individual"])
def test_blend_load_and_commit_match_reference(golden, tag):
    apc, alloc_end, bs, chunk, layers = (int(x) for x in golden[f"loader_{tag}_meta"])
    plan = golden[f"loader_{tag}_plan"]
    slot_mapping = golden[f"loader_{tag}_slot_mapping"][:alloc_end]
    table = oracle.f32_to_bf16(golden[f"loader_{tag}_cos_sin"])
    pages = golden[f"loader_{tag}_pages_before"].copy()
    if tag == "fused":
        moved = any(int(s) != int(t) for s, t, _ in plan)
        rotate = np.full(len(plan), int(moved), dtype=np.int32)
    else:
        rotate = np.array([int(s != t) for s, t, _ in plan], dtype=np.int32)
    for layer in range(layers):
        k = np.ascontiguousarray(pages[layer, 0])
        v = np.ascontiguousarray(pages[layer, 1])
        segments = [
            (int(s), int(t), int(n), golden[f"loader_{tag}_host_{i}_{layer}"])
            for i, (s, t, n) in enumerate(plan)
        ]
        staging = oracle.blend_load(
            BF16, alloc_end, apc, k, v, slot_mapping, bs, segments, rotate, table,
            k.shape[-1], k.shape[-1], True,
        )
        assert np.array_equal(staging, golden[f"loader_{tag}_staging_{layer}"]), layer
        recomputed = golden[f"loader_{tag}_recomputed_{layer}"]
        oracle.paged_scatter(recomputed[:, apc:], k, v, slot_mapping[apc:], bs)
        assert np.array_equal(np.stack([k, v]), golden[f"loader_{tag}_pages_after_{layer}"])


def test_deviation_matches_reference_within_tolerance(golden):
    scores = oracle.kv_deviation(
        golden["dev_fresh"], golden["dev_cached"], BF16, abs_index=golden["dev_absolute"]
    )
    np.testing.assert_allclose(scores, golden["dev_scores"], rtol=1e-5)


@pytest.mark.parametrize("case", range(6))
def test_select_matches_reference(golden, case):
    forced = golden[f"sel_{case}_forced"] if golden[f"sel_{case}_has_forced"][0] else None
    out = oracle.select(
        golden[f"sel_{case}_scores"], golden[f"sel_{case}_gaps"], float(golden[f"sel_{case}_ratio"][0]),
        forced,
    )
    assert np.array_equal(out, golden[f"sel_{case}_out"])


def test_select_known_answers():
    # reference tests/test_ascend.py:144-154 and 256-267
    assert oracle.select(np.array([1.0, 10.0, 2.0, 9.0]), np.array([1, 0, 1, 0], bool), 0.5).tolist() == [0, 1, 2]
    assert oracle.select(
        np.array([0.0, 1.0, 10.0, 9.0]), np.array([1, 0, 0, 0], bool), 0.5,
        forced_mask=np.array([0, 1, 0, 0], bool),
    ).tolist() == [0, 1, 2]


def test_select_ties_keep_lowest_index():
    out = oracle.select(np.array([5.0, 7.0, 7.0, 7.0, 1.0]), np.zeros(5, bool), 0.4)
    assert out.tolist() == [1, 2]


@pytest.mark.parametrize("case", range(3))
def test_sparse_q_matches_reference(golden, case):
    chunk, overflow, tail, block_size = (int(x) for x in golden[f"sq_{case}_meta"])
    query = oracle.bf16_to_f32(golden[f"sq_{case}_query"])
    key = oracle.bf16_to_f32(golden[f"sq_{case}_key"])
    scores, forced, stats = oracle.sparse_q_scores(
        query, key, golden[f"sq_{case}_absolute"], golden[f"sq_{case}_gaps"],
        float(golden[f"sq_{case}_scale"][0]), block_size, overflow, tail, chunk,
    )
    np.testing.assert_allclose(scores, golden[f"sq_{case}_scores"], rtol=1e-4, atol=1e-6)
    assert np.array_equal(forced, golden[f"sq_{case}_forced"])
    expected = golden[f"sq_{case}_stats"]
    assert stats["sparse_query_tokens"] == expected[0]
    assert int(stats["tail_fallback"]) == expected[1]
    selected = oracle.select(scores, golden[f"sq_{case}_gaps"], 0.15, forced)
    assert np.array_equal(selected, golden[f"sq_{case}_selected"])


def test_sparse_q_known_answer_masks():
    # reference tests/test_ascend.py:215-253
    gaps = np.array([False, False, True, False, False, False])
    _, forced, _ = oracle.sparse_q_masks(gaps, 2, 1, 2)
    assert forced.tolist() == [True, True, True, True, True, False]
    query, forced, tail = oracle.sparse_q_masks(np.zeros(6, bool), 2, 1, 2)
    assert forced.tolist() == [False, False, False, False, True, True]
    assert query.sum() == 2 and tail


def test_bf16_rounding_is_nearest_even():
    values = np.array([1.0, 1.00390625, 1.01171875, -3.0e38, np.inf], dtype=np.float32)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 is a tie -> even (1 + 2^-6)
    assert oracle.bf16_to_f32(oracle.f32_to_bf16(values))[:3].tolist() == [1.0, 1.0, 1.015625]
    assert np.isinf(oracle.bf16_to_f32(oracle.f32_to_bf16(values))[-1])


@pytest.mark.parametrize("case", range(2))
def test_sparse_q_head128_matches_reference(golden, case):
    tag = f"sq128_{case}"
    chunk, overflow, tail, block_size = (int(x) for x in golden[f"{tag}_meta"])
    scores, forced, stats = oracle.sparse_q_scores(
        oracle.bf16_to_f32(golden[f"{tag}_query"]), oracle.bf16_to_f32(golden[f"{tag}_key"]),
        golden[f"{tag}_absolute"], golden[f"{tag}_gaps"], float(golden[f"{tag}_scale"][0]), block_size,
        overflow, tail, chunk,
    )
    np.testing.assert_allclose(scores, golden[f"{tag}_scores"], rtol=1e-4, atol=1e-6)
    assert np.array_equal(forced, golden[f"{tag}_forced"])
    assert stats["sparse_query_tokens"] == golden[f"{tag}_stats"][0]
    assert np.array_equal(oracle.select(scores, golden[f"{tag}_gaps"], 0.15, forced), golden[f"{tag}_selected"])


@pytest.mark.parametrize("case", range(3))
def test_attention_matches_reference(attention_golden, case):
    """Oracle attention vs the reference's einsum path (ascend.py:798-846):
    bit-equal except where the fp32 accumulation order flips one rounding of a
    logit or a probability (under 0.5% of the elements, each within 2e-3: one
    probability ulp times a value)."""
    from conftest import element_values

    tag = f"att_{case}"
    code = int(attention_golden[f"{tag}_meta"][0])
    q, k, v = (element_values(attention_golden[f"{tag}_{n}"], code) for n in ("query", "key", "value"))
    got = oracle.blend_attention(q, k, v, attention_golden[f"{tag}_positions"],
                                 float(attention_golden[f"{tag}_scale"][0]), code)
    want = element_values(attention_golden[f"{tag}_out"], code)
    assert (got != want).mean() < 5e-3
    assert float(np.abs(got - want).max()) <= 2e-3
