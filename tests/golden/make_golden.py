"""Generate golden vectors by running the REFERENCE implementation.

    python tests/golden/make_golden.py [--reference /path/to/PIC-KVCache]

Imports the reference package ``cacheblend_vllm`` (pure Python/torch, runs on
CPU) from a read-only checkout and records seeded inputs and its outputs for
the hot-path functions into ``tests/golden/golden.npz``.  The fixtures are
committed; the reference is not needed at test time (and does not exist on
the GPU machines).  bf16 tensors are stored as uint16 bit patterns.

Covered reference functions (file:line in the reference):
  kv_layout.gather_paged_kv / scatter_paged_kv         kv_layout.py:90-161
  ascend.relocate_key (cos_sin_cache branch)          ascend.py:52-103
  ascend.PagedBlendLoader.prefetch/get/commit         ascend.py:224-407
  deviation expression of _compute_layer              ascend.py:535-538
  ascend.Qwen3BlendExecutor._select                   ascend.py:757-796
  ascend.Qwen3BlendExecutor._sparse_q_scores          ascend.py:638-711
  storage.LocalPinnedCPUStore (op sequence)           storage.py:56-294
  hashing.content_hash / rolling_hash_values          hashing.py:18-53  (hashes.npz)
  ascend.Qwen3BlendExecutor._attention (einsum path)  ascend.py:798-846 (attention.npz)
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden.npz"
STORE_OUT = Path(__file__).resolve().parent / "store_sequence.json"
HASH_OUT = Path(__file__).resolve().parent / "hashes.npz"
ATTENTION_OUT = Path(__file__).resolve().parent / "attention.npz"


def make_hash_golden() -> None:
    """Reference fingerprints (hashing.py:18-53): every 256-token window of a seeded prompt
    (token ids up to 2**31 and a negative one) and the content hash of each chunk."""
    from cacheblend_vllm.hashing import content_hash, rolling_hash_values

    rng = np.random.default_rng(31)
    tokens = rng.integers(0, 151_936, size=4096).astype(np.int64)
    tokens[[5, 700, 3000]] = [2**31 - 1, 0, 123_456_789]
    windows = rolling_hash_values(tokens.tolist(), 256)
    chunks = np.array([content_hash(tokens[i : i + 256].tolist()) for i in range(0, 4096, 256)],
                      dtype=np.uint64)
    small = np.array([content_hash([7]), content_hash([-1, 0, 1]), content_hash([])], dtype=np.uint64)
    np.savez_compressed(HASH_OUT, tokens=tokens, windows=windows, chunks=chunks, small=small)


def make_attention_golden() -> None:
    """The reference's attention of computed queries over the staging context
    (ascend.py:798-846), CPU einsum path, head size 128: pruned and prefill
    positions, query groups 4 / 1 / 8, bf16 and fp16."""
    from types import SimpleNamespace

    from cacheblend_vllm.ascend import Qwen3BlendExecutor
    from cacheblend_vllm.config import CacheBlendConfig

    gen = torch.Generator().manual_seed(41)
    gold = {}
    for case, (nq, nk, hq, hkv, dtype, pruned) in enumerate(
        [(64, 300, 8, 2, torch.bfloat16, True), (130, 130, 4, 4, torch.bfloat16, False),
         (33, 200, 8, 1, torch.float16, True)]
    ):
        executor = object.__new__(Qwen3BlendExecutor)
        executor.config = CacheBlendConfig.from_extra_config({"strict_version_check": False})
        if pruned:
            pick = torch.randperm(nk - 1, generator=gen)[: nq - 1].sort().values
            positions = torch.cat([pick, torch.tensor([nk - 1])])
        else:
            positions = torch.arange(nk - nq, nk)
        query = torch.randn(nq, hq, 128, generator=gen).to(dtype)
        key = torch.randn(nk, hkv, 128, generator=gen).to(dtype)
        value = torch.randn(nk, hkv, 128, generator=gen).to(dtype)
        scale = 1.0 / math.sqrt(128)
        state = SimpleNamespace(important_indices=None, attention_mask=None)
        out = executor._attention(query, key, value, positions, scale, state)
        as_bits = bits if dtype == torch.bfloat16 else (lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16).copy())
        tag = f"att_{case}"
        gold[f"{tag}_query"] = as_bits(query)
        gold[f"{tag}_key"] = as_bits(key)
        gold[f"{tag}_value"] = as_bits(value)
        gold[f"{tag}_positions"] = positions.numpy()
        gold[f"{tag}_meta"] = np.array([0 if dtype == torch.bfloat16 else 1], dtype=np.int64)
        gold[f"{tag}_scale"] = np.array([scale])
        gold[f"{tag}_out"] = as_bits(out)
    np.savez_compressed(ATTENTION_OUT, **gold)


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.contiguous().numpy().copy()


class Rope:
    """vLLM-style rotary module: fp32 cos_sin_cache [max_pos, rotary_dim]."""

    def __init__(self, head_size: int, rotary_dim: int, max_pos: int, base: float, neox: bool):
        self.head_size = head_size
        self.rotary_dim = rotary_dim
        self.is_neox_style = neox
        inv = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim))
        freqs = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos_sin_cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("CACHEBLEND_REFERENCE"),
                        help="checkout of the reference (the directory holding cacheblend_vllm/); "
                             "or set CACHEBLEND_REFERENCE")
    args = parser.parse_args()
    if not args.reference:
        parser.error("pass --reference <checkout> or set CACHEBLEND_REFERENCE")
    sys.path.insert(0, args.reference)
    sys.dont_write_bytecode = True
    from cacheblend_vllm.ascend import PagedBlendLoader, Qwen3BlendExecutor, relocate_key
    from cacheblend_vllm.config import CacheBlendConfig
    from cacheblend_vllm.kv_layout import gather_paged_kv, scatter_paged_kv
    from cacheblend_vllm.storage import LocalPinnedCPUStore
    from cacheblend_vllm.types import BlendPlan, BlendSegment

    gold: dict[str, np.ndarray] = {}
    gen = torch.Generator().manual_seed(1234)

    # ---- 1. paged gather / scatter, three layouts, bf16 [NB=6, BS=4, H=2, D=16]
    nb, bs, h, d = 6, 4, 2, 16
    base = torch.randn(2, nb, bs, h, d, generator=gen).to(torch.bfloat16)
    slots = torch.tensor([0, 5, 23, 7, 12, -1, 3, 18], dtype=torch.long)
    replacement = torch.randn(2, slots.numel(), h, d, generator=gen).to(torch.bfloat16)
    gold["kv_base"] = bits(base)
    gold["kv_slots"] = slots.numpy()
    gold["kv_replacement"] = bits(replacement)
    for layout in ("merged_first", "merged_block", "separate"):
        if layout == "merged_first":
            paged = base.clone()
        elif layout == "merged_block":
            paged = base.permute(1, 0, 2, 3, 4).contiguous()
        else:
            paged = [base[0].clone(), base[1].clone()]
        gathered = gather_paged_kv(paged, slots, bs)
        gold[f"kv_gather_{layout}"] = bits(gathered)
        scatter_paged_kv(replacement[:, :5], paged, slots[:5], bs)
        after = paged if isinstance(paged, torch.Tensor) else torch.stack(paged)
        if layout == "merged_block":
            after = after.permute(1, 0, 2, 3, 4)
        gold[f"kv_scatter_{layout}"] = bits(after.contiguous())

    # ---- 2. relocate_key: bf16 neox / GPT-J (head 64, rotary 64), fp32 neox
    for name, dtype, neox, rot in (
        ("bf16_neox", torch.bfloat16, True, 64),
        ("bf16_gptj", torch.bfloat16, False, 64),
        ("fp32_neox", torch.float32, True, 64),
        ("bf16_partial", torch.bfloat16, True, 32),
    ):
        rope = Rope(64, rot, 1024, 1e6, neox)
        key = torch.randn(37, 3 * 64, generator=gen).to(dtype)
        old = torch.randint(0, 1024, (37,), generator=gen)
        new = torch.randint(0, 1024, (37,), generator=gen)
        old[:3] = new[:3]  # identity positions are still rotated (bits may move)
        out = relocate_key(rope, old, new, key)
        gold[f"rope_{name}_key"] = bits(key)
        gold[f"rope_{name}_cos_sin"] = rope.cos_sin_cache.numpy()
        gold[f"rope_{name}_old"] = old.numpy()
        gold[f"rope_{name}_new"] = new.numpy()
        gold[f"rope_{name}_out"] = bits(out)

    # ---- 3. PagedBlendLoader: APC prefix, gaps, relocated non-contiguous hits
    for fused in (True, False):
        tag = "fused" if fused else "individual"
        chunk, layers, h2, d2, bs2, nb2 = 8, 2, 2, 32, 4, 24
        config = CacheBlendConfig.from_extra_config(
            {"chunk_size": chunk, "local_cpu_gb": 0.01, "event_pipeline": False,
             "strict_version_check": False, "fused_segment_copy": fused}
        )
        store = LocalPinnedCPUStore(chunk, 1 << 24, pin_memory=False)
        pages = [torch.randn(2, nb2, bs2, h2, d2, generator=gen).to(torch.bfloat16) for _ in range(layers)]
        gold[f"loader_{tag}_pages_before"] = np.stack([bits(page) for page in pages])
        perm = torch.randperm(nb2, generator=gen)
        block_ids = perm[:12].tolist()
        slot_mapping = (torch.tensor(block_ids)[:, None] * bs2 + torch.arange(bs2)[None, :]).flatten()
        apc = 4
        targets = [8, 24, 32]  # gaps at [4, 8), [16, 24)
        sources = [40, 24, 100]  # second hit not relocated
        segments = []
        hosts = {}
        for i, (src, tgt) in enumerate(zip(sources, targets)):
            tokens = list(range(1000 * (i + 1), 1000 * (i + 1) + chunk))
            sid = store.begin_put("m", src, tokens, layers)
            for layer in range(layers):
                parent = torch.randn(2, 3 * chunk, h2, d2, generator=gen).to(torch.bfloat16)
                view = parent[:, chunk : 2 * chunk]  # non-contiguous published view
                store.put_layer_host(sid, layer, view)
                hosts[(i, layer)] = view.contiguous()
            segments.append(BlendSegment(sid, tgt))
        store.pin("r", segments)
        plan = BlendPlan.from_segments(apc, segments)
        rope = Rope(d2, d2, 256, 1e4, True)
        loader = PagedBlendLoader(pages, store, "r", plan, slot_mapping, bs2, config)
        for layer in range(layers):
            loader.prefetch(layer, rope)
            staging = loader.get(layer)
            gold[f"loader_{tag}_staging_{layer}"] = bits(staging)
            recomputed = staging.clone()
            recomputed[:, apc:] = torch.randn(recomputed[:, apc:].shape, generator=gen).to(torch.bfloat16)
            gold[f"loader_{tag}_recomputed_{layer}"] = bits(recomputed)
            loader.commit(layer, recomputed)
            gold[f"loader_{tag}_pages_after_{layer}"] = bits(pages[layer])
        for i in range(len(segments)):
            for layer in range(layers):
                gold[f"loader_{tag}_host_{i}_{layer}"] = bits(hosts[(i, layer)])
        gold[f"loader_{tag}_cos_sin"] = rope.cos_sin_cache.numpy()
        gold[f"loader_{tag}_slot_mapping"] = slot_mapping.numpy()
        gold[f"loader_{tag}_plan"] = np.array(
            [[s, t, chunk] for s, t in zip(sources, targets)], dtype=np.int64
        )
        gold[f"loader_{tag}_meta"] = np.array([apc, plan.allocation_end, bs2, chunk, layers], dtype=np.int64)

    # ---- 4. deviation expression (ascend.py:535-538) on bf16
    k_fresh = torch.randn(50, 256, generator=gen).to(torch.bfloat16)
    flat_old = torch.randn(70, 256, generator=gen).to(torch.bfloat16)
    absolute = torch.arange(10, 60)
    dev = torch.sum((k_fresh.float() - flat_old[absolute].float()) ** 2, dim=-1)
    gold["dev_fresh"] = bits(k_fresh)
    gold["dev_cached"] = bits(flat_old)
    gold["dev_absolute"] = absolute.numpy()
    gold["dev_scores"] = dev.numpy()

    # ---- 5. _select
    executor = object.__new__(Qwen3BlendExecutor)
    executor.tp_group = None
    cases = []
    for case in range(6):
        n = [1, 4, 57, 300, 1000, 33][case]
        ratio = [0.15, 0.5, 0.15, 0.3, 0.0, 1.0][case]
        executor.config = CacheBlendConfig.from_extra_config(
            {"recompute_ratios": [ratio], "strict_version_check": False}
        )
        scores = torch.rand(n, generator=gen) * 10
        gaps = torch.rand(n, generator=gen) < 0.3
        forced = (torch.rand(n, generator=gen) < 0.1) if case % 2 else None
        selected = executor._select(scores, gaps, forced_mask=forced)
        gold[f"sel_{case}_scores"] = scores.numpy()
        gold[f"sel_{case}_gaps"] = gaps.numpy()
        gold[f"sel_{case}_forced"] = (forced if forced is not None else torch.zeros(n, dtype=torch.bool)).numpy()
        gold[f"sel_{case}_has_forced"] = np.array([forced is not None])
        gold[f"sel_{case}_ratio"] = np.array([ratio])
        gold[f"sel_{case}_out"] = selected.numpy()
        cases.append(case)

    # ---- 6. _sparse_q_scores (bf16 Q/K, groups 4)
    for case, (active, ctx, hq, hkv, chunk_q, overflow, gap_spans) in enumerate(
        [
            (40, 52, 8, 2, 8, 1, [(5, 9), (30, 40)]),
            (24, 24, 4, 1, 3, 0, [(0, 2), (20, 24)]),
            (16, 30, 4, 2, 8, 2, []),  # tail fallback
        ]
    ):
        executor = object.__new__(Qwen3BlendExecutor)
        executor.tp_group = None
        executor.block_size = 4
        executor.config = CacheBlendConfig.from_extra_config(
            {"selection_strategy": "sparse_q", "check_layers": [1], "query_score_chunk_size": chunk_q,
             "overflow_blocks": overflow, "tail_query_tokens": 6, "strict_version_check": False}
        )
        query = torch.randn(active, hq, 32, generator=gen).to(torch.bfloat16)
        key = torch.randn(ctx, hkv, 32, generator=gen).to(torch.bfloat16)
        compute_start = ctx - active
        absolute = torch.arange(compute_start, ctx)
        gaps = torch.zeros(active, dtype=torch.bool)
        for a, b in gap_spans:
            gaps[a:b] = True
        scale = 1.0 / math.sqrt(32)
        scores, forced, stats = executor._sparse_q_scores(query, key, absolute, gaps, scale)
        selected = executor._select(scores, gaps, 1, forced_mask=forced)
        gold[f"sq_{case}_query"] = bits(query)
        gold[f"sq_{case}_key"] = bits(key)
        gold[f"sq_{case}_absolute"] = absolute.numpy()
        gold[f"sq_{case}_gaps"] = gaps.numpy()
        gold[f"sq_{case}_meta"] = np.array([chunk_q, overflow, 6, 4], dtype=np.int64)
        gold[f"sq_{case}_scale"] = np.array([scale])
        gold[f"sq_{case}_scores"] = scores.numpy()
        gold[f"sq_{case}_forced"] = forced.numpy()
        gold[f"sq_{case}_selected"] = selected.numpy()
        gold[f"sq_{case}_stats"] = np.array(
            [stats["sparse_query_tokens"], int(stats["tail_fallback"]), stats["gap_tokens"]], dtype=np.int64
        )

    # ---- 6b. _sparse_q_scores at the real head size (128), bf16
    for case, (active, ctx, hq, hkv, chunk_q, overflow, gap_spans, tail) in enumerate(
        [
            (300, 400, 8, 2, 8, 1, [(20, 60), (200, 260)], 64),
            (200, 200, 16, 2, 8, 1, [], 64),  # tail fallback, no prefix
        ]
    ):
        executor = object.__new__(Qwen3BlendExecutor)
        executor.tp_group = None
        executor.block_size = 16
        executor.config = CacheBlendConfig.from_extra_config(
            {"selection_strategy": "sparse_q", "check_layers": [1], "query_score_chunk_size": chunk_q,
             "overflow_blocks": overflow, "tail_query_tokens": tail, "recompute_ratios": [0.15],
             "strict_version_check": False}
        )
        query = torch.randn(active, hq, 128, generator=gen).to(torch.bfloat16)
        key = torch.randn(ctx, hkv, 128, generator=gen).to(torch.bfloat16)
        absolute = torch.arange(ctx - active, ctx)
        gaps = torch.zeros(active, dtype=torch.bool)
        for a, b in gap_spans:
            gaps[a:b] = True
        scale = 1.0 / math.sqrt(128)
        scores, forced, stats = executor._sparse_q_scores(query, key, absolute, gaps, scale)
        selected = executor._select(scores, gaps, 1, forced_mask=forced)
        tag = f"sq128_{case}"
        gold[f"{tag}_query"] = bits(query)
        gold[f"{tag}_key"] = bits(key)
        gold[f"{tag}_absolute"] = absolute.numpy()
        gold[f"{tag}_gaps"] = gaps.numpy()
        gold[f"{tag}_meta"] = np.array([chunk_q, overflow, tail, 16], dtype=np.int64)
        gold[f"{tag}_scale"] = np.array([scale])
        gold[f"{tag}_scores"] = scores.numpy()
        gold[f"{tag}_forced"] = forced.numpy()
        gold[f"{tag}_selected"] = selected.numpy()
        gold[f"{tag}_stats"] = np.array(
            [stats["sparse_query_tokens"], int(stats["tail_fallback"]), stats["gap_tokens"]], dtype=np.int64
        )

    np.savez_compressed(OUT, **gold)
    make_hash_golden()
    make_attention_golden()

    # ---- 7. store op sequence: every call, its result, bytes and LRU order
    rng = np.random.default_rng(7)
    store = LocalPinnedCPUStore(4, max_bytes=10 * 2 * 4 * 2 * 4, pin_memory=False)
    log = []
    known: list = []  # [(segment_id, tokens, source)]

    def order() -> list[int]:
        ids = [entry[0] for entry in known]
        return [ids.index(sid) for sid in store._entries]

    for _ in range(500):
        op = str(rng.choice(["begin", "put", "reserve", "cancel", "abort", "pin", "release", "match"],
                            p=[0.2, 0.3, 0.1, 0.05, 0.05, 0.1, 0.1, 0.1]))
        if op == "begin" or not known:
            base_tok = int(rng.integers(0, 12)) * 10
            tokens = list(range(base_tok, base_tok + 4))
            source = int(rng.integers(0, 4)) * 4
            sid = store.begin_put("m", source, tokens, 2)
            if all(entry[0] != sid for entry in known):
                known.append((sid, tokens, source))
            record = {"op": "begin", "source": source, "tokens": tokens}
        else:
            index = int(rng.integers(0, len(known)))
            sid, tokens, _ = known[index]
            record = {"op": op, "index": index}
            if op == "put":
                record["layer"] = int(rng.integers(0, 2))
                record["width"] = int(rng.choice([2, 2, 3]))
                record["result"] = store.put_layer_host(sid, record["layer"], torch.zeros(2, 4, record["width"]))
            elif op == "reserve":
                record["layer"] = int(rng.integers(0, 2))
                record["result"] = store.reserve_layer(sid, record["layer"])
            elif op == "cancel":
                record["layer"] = int(rng.integers(0, 2))
                store.cancel_layer(sid, record["layer"])
            elif op == "abort":
                store.abort_put(sid)
            elif op == "pin":
                record["request"] = f"r{int(rng.integers(0, 3))}"
                record["indices"] = [int(j) for j in rng.choice(len(known), size=min(2, len(known)), replace=False)]
                segs = [BlendSegment(known[j][0], 0) for j in record["indices"]]
                ids = [entry[0] for entry in known]
                record["result"] = [ids.index(seg.segment_id) for seg in store.pin(record["request"], segs)]
            elif op == "release":
                record["request"] = f"r{int(rng.integers(0, 3))}"
                store.release(record["request"])
            else:
                ids = [entry[0] for entry in known]
                record["result"] = [ids.index(seg.segment_id) for seg in store.match("m", tokens, 0)]
        record["bytes"] = store.current_bytes
        record["committed"] = store.committed_entries
        record["order"] = order()
        log.append(record)
    STORE_OUT.write_text(json.dumps({"max_bytes": store.max_bytes, "chunk": 4, "log": log}))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes) and {STORE_OUT}")


if __name__ == "__main__":
    main()
