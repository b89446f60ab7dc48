"""The layerwise side executor (Qwen3BlendExecutor._compute_layer,
cacheblend_vllm/ascend.py:487-630) driven with small stand-in Qwen3 layers on
the GPU: a plain layer and a check layer under each selection strategy
(kv_deviation, sparse_q, compare).  The executor's seams (K-deviation score,
Sparse-Q score, select, staging write-back, attention over the staging) run on
the sm_100a kernels; the expectation restates the reference's layer in torch
with the oracle's deviation, Sparse-Q and select and the reference's attention
formula.  Selected indices and the staging bytes must match exactly (Sparse-Q:
except ties within its 1e-3 tolerance); hidden states within the attention
tolerance (bf16 products downstream).  A last test runs Qwen3BlendExecutor.run
end to end through PagedBlendLoader (store -> H2D -> relocation -> layers ->
commit) and compares the pages bit for bit."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.attention import blend_attention
from cacheblend_b200.config import CacheBlendConfig
from cacheblend_b200.executor import BlendExecutionState, Qwen3BlendExecutor

pytestmark = pytest.mark.gpu

HIDDEN, HQ, HKV, HD, INTER = 256, 4, 2, 128, 384


class _Norm:
    """vLLM RMSNorm calling convention: norm(x) or norm(x, residual) -> (norm(x + r), x + r)."""

    def __init__(self, dim, gen, device):
        self.w = (1.0 + 0.1 * torch.randn(dim, generator=gen)).to(device)

    def _apply(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * self.w).to(x.dtype)

    def __call__(self, x, residual=None):
        if residual is None:
            return self._apply(x)
        s = x + residual
        return self._apply(s), s


class _Linear:
    def __init__(self, out_dim, in_dim, gen, device):
        self.w = (torch.randn(out_dim, in_dim, generator=gen) * in_dim ** -0.5).to(torch.bfloat16).to(device)

    def __call__(self, x):
        return x @ self.w.t(), None


class _Mlp:
    def __init__(self, gen, device):
        self.up = _Linear(INTER, HIDDEN, gen, device)
        self.down = _Linear(HIDDEN, INTER, gen, device)

    def __call__(self, x):
        return self.down(torch.nn.functional.silu(self.up(x)[0]))[0]


class _Rope:
    """NeoX rotary over the full head with vLLM's cos_sin_cache layout."""

    def __init__(self, max_pos, device):
        inv = 1.0 / (1e6 ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD))
        freqs = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos_sin_cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(device)
        self.head_size, self.rotary_dim, self.is_neox_style = HD, HD, True

    def _rotate(self, x, positions):
        shape = x.shape
        x = x.view(x.shape[0], -1, HD).float()
        cos, sin = self.cos_sin_cache[positions].chunk(2, dim=-1)
        cos, sin = cos[:, None, :], sin[:, None, :]
        x1, x2 = x[..., : HD // 2], x[..., HD // 2 :]
        out = torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)
        return out.to(torch.bfloat16).reshape(shape)

    def __call__(self, positions, q, k):
        return self._rotate(q, positions), self._rotate(k, positions)


def _layer(gen, device, max_pos):
    attn = SimpleNamespace(num_heads=HQ, num_kv_heads=HKV, head_size=HD,
                           impl=SimpleNamespace(scale=HD ** -0.5))
    self_attn = SimpleNamespace(
        qkv_proj=_Linear((HQ + 2 * HKV) * HD, HIDDEN, gen, device), q_size=HQ * HD, kv_size=HKV * HD,
        head_dim=HD, q_norm=_Norm(HD, gen, device), k_norm=_Norm(HD, gen, device),
        rotary_emb=_Rope(max_pos, device), attn=attn, o_proj=_Linear(HIDDEN, HQ * HD, gen, device))
    return SimpleNamespace(input_layernorm=_Norm(HIDDEN, gen, device), self_attn=self_attn,
                           post_attention_layernorm=_Norm(HIDDEN, gen, device), mlp=_Mlp(gen, device))


def _reference_attention(query, key, value, positions, scale):
    groups = HQ // HKV
    masked = positions[:, None] < torch.arange(key.shape[0], device=query.device)[None, :]
    out = torch.empty_like(query)
    for h in range(HKV):
        q = query[:, h * groups:(h + 1) * groups]
        w = torch.einsum("qgd,kd->gqk", q, key[:, h]) * scale
        w = w.masked_fill(masked[None], torch.finfo(w.dtype).min)
        p = torch.softmax(w.float(), dim=-1).to(query.dtype)
        out[:, h * groups:(h + 1) * groups] = torch.einsum("gqk,kd->qgd", p, value[:, h])
    return out


def _reference_layer(layer, hidden, residual, positions, old_kv, compute_start, gap_mask, check, ratio,
                     attention=_reference_attention):
    """ascend.py:487-630 for one layer, kv_deviation strategy, in torch + oracle."""
    sa = layer.self_attn
    if residual is None:
        residual = hidden
        hidden = layer.input_layernorm(hidden)
    else:
        hidden, residual = layer.input_layernorm(hidden, residual)
    qkv, _ = sa.qkv_proj(hidden)
    q, k, v = qkv.split([sa.q_size, sa.kv_size, sa.kv_size], dim=-1)
    q = sa.q_norm(q.view(-1, HQ, HD)).view(q.shape)
    k = sa.k_norm(k.view(-1, HKV, HD)).view(k.shape)
    q, k = sa.rotary_emb(positions, q, k)
    query_indices = torch.arange(q.shape[0], device=q.device)
    absolute = compute_start + query_indices
    flat_k = old_kv[0].reshape(old_kv.shape[1], -1)
    flat_v = old_kv[1].reshape(old_kv.shape[1], -1)
    selected = None
    if check:
        bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        scores = oracle.kv_deviation(bits(k), bits(flat_k), oracle.BF16, absolute.cpu().numpy())
        gaps = gap_mask[absolute.cpu().numpy()]
        selected = torch.from_numpy(oracle.select(scores, gaps, ratio)).to(q.device)
        q, k, v, residual = q[selected], k[selected], v[selected], residual[selected]
        absolute = compute_start + selected
        positions = positions[selected]
    flat_k[absolute] = k
    flat_v[absolute] = v
    out = attention(q.view(-1, HQ, HD), old_kv[0].view(-1, HKV, HD), old_kv[1].view(-1, HKV, HD),
                    absolute, sa.attn.impl.scale).reshape(-1, HQ * HD)
    hidden, _ = sa.o_proj(out)
    hidden, residual = layer.post_attention_layernorm(hidden, residual)
    return layer.mlp(hidden), residual, positions, selected


def test_executor_layers_match_reference(cuda):
    gen = torch.Generator().manual_seed(8)
    ctx, compute_start = 520, 40  # staging rows [0, 520), tokens computed from position 40
    n = ctx - compute_start
    layers = [_layer(gen, cuda, ctx), _layer(gen, cuda, ctx)]
    executor = object.__new__(Qwen3BlendExecutor)
    executor.config = CacheBlendConfig.from_extra_config(
        {"check_layers": [1], "recompute_ratios": [0.15], "selection_strategy": "kv_deviation",
         "strict_version_check": False})
    executor.block_size = 16
    executor.tp_group = None
    executor.layers = layers
    gap_mask = np.zeros(ctx, dtype=bool)
    gap_mask[200:260] = True
    gap_mask[ctx - 1] = True
    hidden = (torch.randn(n, HIDDEN, generator=gen) * 0.5).to(torch.bfloat16).to(cuda)
    staging = [(torch.randn(2, ctx, HKV, HD, generator=gen)).to(torch.bfloat16).to(cuda) for _ in layers]
    ref_staging = [s.clone() for s in staging]

    state = BlendExecutionState(compute_start, torch.arange(compute_start, ctx, device=cuda), gap_mask)
    h, r = hidden, None
    ref_h, ref_r, ref_pos = hidden, None, torch.arange(compute_start, ctx, device=cuda)
    for layer_id, layer in enumerate(layers):
        h, r, state, staging[layer_id] = executor._compute_layer(layer_id, layer, h, r, state, staging[layer_id])
        ref_h, ref_r, ref_pos, selected = _reference_layer(
            layer, ref_h, ref_r, ref_pos, ref_staging[layer_id], compute_start, gap_mask,
            check=layer_id == 1, ratio=0.15)
        if selected is not None:
            assert torch.equal(state.important_indices, selected)
            assert torch.equal(state.positions, ref_pos)
        # staging after the write-back: fresh K/V rows of the computed tokens (bit-exact)
        assert torch.equal(staging[layer_id], ref_staging[layer_id]), layer_id
        diff = (h.float() - ref_h.float()).abs()
        assert float(diff.max()) <= 5e-2 + 5e-2 * float(ref_h.float().abs().max()), layer_id
        assert float(diff.mean()) <= 5e-3, layer_id
        # continue both from the same values so the next layer compares like with like
        ref_h, ref_r = h, r
    assert h.shape[0] == state.important_indices.numel()


class _Tracer:
    enabled = True

    def __init__(self):
        self.events = []

    def emit(self, name, **fields):
        self.events.append((name, fields))


def _executor(layers, strategy):
    executor = object.__new__(Qwen3BlendExecutor)
    executor.config = CacheBlendConfig.from_extra_config(
        {"check_layers": [1], "recompute_ratios": [0.15], "selection_strategy": strategy,
         "strict_version_check": False})
    executor.block_size = 16
    executor.tp_group = None
    executor.layers = layers
    return executor


def _close_selection(got, want, scores, gaps, forced, ratio=0.15):
    """Index sets equal, or differing only at scores tied with the threshold within 1e-3."""
    if np.array_equal(got, want):
        return
    diff = np.setxor1d(got, want)
    base = gaps | forced
    candidates = np.flatnonzero(~base)
    k = len(want) - int(base.sum())
    threshold = np.sort(scores[candidates])[::-1][k - 1]
    assert np.all(np.abs(scores[diff] - threshold) <= 1e-3 * abs(threshold)), diff


@pytest.mark.parametrize("strategy", ["sparse_q", "compare"])
def test_executor_query_aware_strategies(cuda, strategy):
    """sparse_q: score the check layer's queries against the staged keys (fresh
    keys written in place) on the tensor cores, attend with every row, prune
    after the MLP; compare: prune by K-deviation exactly as kv_deviation does
    and report the overlap of the two selections (ascend.py:545-630)."""
    gen = torch.Generator().manual_seed(9)
    ctx, compute_start = 700, 60
    n = ctx - compute_start
    layers = [_layer(gen, cuda, ctx), _layer(gen, cuda, ctx)]
    gap_mask = np.zeros(ctx, dtype=bool)
    gap_mask[300:380] = True
    gap_mask[ctx - 1] = True
    hidden = (torch.randn(n, HIDDEN, generator=gen) * 0.5).to(torch.bfloat16).to(cuda)
    staging0 = [torch.randn(2, ctx, HKV, HD, generator=gen).to(torch.bfloat16).to(cuda) for _ in layers]

    def run(strategy_name, tracer=None):
        executor = _executor(layers, strategy_name)
        staging = [s.clone() for s in staging0]
        state = BlendExecutionState(compute_start, torch.arange(compute_start, ctx, device=cuda), gap_mask)
        h, r = hidden, None
        for layer_id, layer in enumerate(layers):
            h, r, state, staging[layer_id] = executor._compute_layer(
                layer_id, layer, h, r, state, staging[layer_id], request_id="req", tracer=tracer)
        return h, r, state, staging

    if strategy == "sparse_q":
        h, r, state, staging = run("sparse_q")
        # expectation: layer 0 as before, then layer 1 with every row and oracle Sparse-Q
        executor = _executor(layers, "kv_deviation")
        ref_staging = [s.clone() for s in staging0]
        ref_state = BlendExecutionState(compute_start, torch.arange(compute_start, ctx, device=cuda), gap_mask)
        h0, r0, ref_state, ref_staging[0] = executor._compute_layer(0, layers[0], hidden, None, ref_state,
                                                                    ref_staging[0])
        assert torch.equal(staging[0], ref_staging[0])
        sa = layers[1].self_attn
        hh, rr = layers[1].input_layernorm(h0, r0)
        qkv, _ = sa.qkv_proj(hh)
        q, k, v = qkv.split([sa.q_size, sa.kv_size, sa.kv_size], dim=-1)
        q = sa.q_norm(q.view(-1, HQ, HD)).view(q.shape)
        k = sa.k_norm(k.view(-1, HKV, HD)).view(k.shape)
        positions = torch.arange(compute_start, ctx, device=cuda)
        q, k = sa.rotary_emb(positions, q, k)
        absolute = np.arange(compute_start, ctx)
        score_keys = ref_staging[1][0].reshape(ctx, -1).clone()
        score_keys[torch.from_numpy(absolute).to(cuda)] = k
        gaps = gap_mask[absolute]
        cfg = executor.config
        want_scores, want_forced, _ = oracle.sparse_q_scores(
            q.view(-1, HQ, HD).float().cpu().numpy(), score_keys.view(ctx, HKV, HD).float().cpu().numpy(),
            absolute, gaps, HD ** -0.5, 16, cfg.overflow_blocks, cfg.tail_query_tokens)
        want_sel = oracle.select(want_scores, gaps, 0.15, want_forced)
        got_sel = state.important_indices.cpu().numpy()
        _close_selection(got_sel, want_sel, want_scores, gaps, want_forced)
        assert h.shape[0] == got_sel.size and r.shape[0] == got_sel.size
        # the staging holds every row's fresh K / V (no pruning before attention)
        flat_k = ref_staging[1][0].reshape(ctx, -1)
        flat_k[torch.from_numpy(absolute).to(cuda)] = k
        assert torch.equal(staging[1][0].reshape(ctx, -1), flat_k)
    else:
        tracer = _Tracer()
        h, r, state, staging = run("compare", tracer)
        h_dev, r_dev, state_dev, staging_dev = run("kv_deviation")
        assert torch.equal(state.important_indices, state_dev.important_indices)
        assert torch.equal(h, h_dev) and torch.equal(r, r_dev)
        assert all(torch.equal(a, b) for a, b in zip(staging, staging_dev))
        events = [f for name, f in tracer.events if name == "selection_compared"]
        assert len(events) == 1
        event = events[0]
        assert event["deviation_tokens"] == state_dev.important_indices.numel()
        sq_sel = run("sparse_q")[2].important_indices.cpu().numpy()
        overlap = np.intersect1d(sq_sel, state_dev.important_indices.cpu().numpy()).size
        assert event["overlap_tokens"] == overlap


def test_executor_run_through_the_loader(cuda):
    """Qwen3BlendExecutor.run end to end (ascend.py:443-485): the loader stages
    the APC prefix from the pages and two stored chunks relocated from other
    positions, the executor computes both layers (kv_deviation at layer 1) and
    the loader commits the span into the pages.  The pages afterwards must equal,
    bit for bit, the oracle's staging of each layer overwritten with the
    reference layer's fresh K/V rows."""
    from cacheblend_b200.loader import PagedBlendLoader
    from cacheblend_b200.storage import LocalPinnedCPUStore
    from cacheblend_b200.types import BlendPlan, BlendSegment

    gen = torch.Generator().manual_seed(10)
    chunk, bs, pool, apc = 64, 16, 64, 64
    hits = [(400, 128), (64, 320)]  # (source_start, target_start)
    max_pos = 1024
    layers = [_layer(gen, cuda, max_pos), _layer(gen, cuda, max_pos)]
    embed = (torch.randn(1000, HIDDEN, generator=gen) * 0.5).to(torch.bfloat16).to(cuda)
    model = SimpleNamespace(model=SimpleNamespace(layers=layers, start_layer=0, end_layer=len(layers),
                                                  embed_tokens=lambda ids: embed[ids]))
    config = CacheBlendConfig.from_extra_config(
        {"chunk_size": chunk, "check_layers": [1], "recompute_ratios": [0.15],
         "selection_strategy": "kv_deviation", "strict_version_check": False})
    executor = _executor(layers, "kv_deviation")
    executor.model = model
    executor.config = config
    pages = [torch.randn(2, pool, bs, HKV, HD, generator=gen).to(torch.bfloat16).to(cuda) for _ in layers]
    before = [p.clone() for p in pages]
    tokens = torch.randint(0, 1000, (400,), generator=gen).tolist()
    blocks = torch.randperm(pool, generator=gen)[:25]
    slots = (blocks[:, None] * bs + torch.arange(bs)[None, :]).reshape(-1)[:400]
    store = LocalPinnedCPUStore(chunk, 1 << 26)
    chunk_data = {}
    segments = []
    for source, target in hits:
        sid = store.begin_put("scope", source, tokens[target : target + chunk], len(layers))
        for layer in range(len(layers)):
            host = torch.randn(2, chunk, HKV, HD, generator=gen).to(torch.bfloat16).pin_memory()
            chunk_data[(sid, layer)] = host
            store.put_layer_host(sid, layer, host)
        segments.append(BlendSegment(sid, target))
    plan = BlendPlan.from_segments(apc, segments)
    assert store.pin("req", segments) == tuple(sorted(segments, key=lambda s: s.target_start))
    loader = PagedBlendLoader(pages, store, "req", plan, slots, bs, config, load_stream=torch.cuda.Stream(cuda))
    executor.run("req", tokens, plan, loader)
    torch.cuda.synchronize()

    # expectation, layer by layer
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    end = plan.allocation_end
    n = end - apc
    gap_mask = plan.gap_mask()
    hidden, residual = embed[torch.tensor(tokens[apc:end], device=cuda)], None
    positions = torch.arange(apc, end, device=cuda)
    slot_np = slots[:end].numpy()
    for layer_id, layer in enumerate(layers):
        k_cache = bits(before[layer_id][0])
        v_cache = bits(before[layer_id][1])
        table = oracle.f32_to_bf16(layer.self_attn.rotary_emb.cos_sin_cache.cpu().numpy())
        segs = [(seg.segment_id.source_start, seg.target_start, chunk, bits(chunk_data[(seg.segment_id, layer_id)]))
                for seg in plan.segments]
        staged = oracle.blend_load(oracle.BF16, end, apc, k_cache, v_cache, slot_np, bs, segs,
                                   np.ones(len(segs), dtype=np.int32), table, HD, HD, True)
        staging = torch.from_numpy(staged.view(np.int16)).view(torch.bfloat16).to(cuda)
        # the attention itself is checked elsewhere; here the same kernel keeps the
        # downstream rows bit-identical so the pages can be compared exactly
        hidden, residual, positions, _ = _reference_layer(
            layer, hidden, residual, positions, staging, apc, gap_mask, check=layer_id == 1, ratio=0.15,
            attention=lambda q, k, v, pos, scale: blend_attention(q, k, v, pos, scale))
        want = before[layer_id].clone()
        flat = want.view(2, pool * bs, HKV, HD)
        idx = torch.from_numpy(slot_np[apc:end]).to(cuda)
        flat[:, idx] = staging[:, apc:end]
        assert torch.equal(pages[layer_id], want), layer_id
