"""Every code path of cb_blend_load_layer against the oracle, bit for bit:
the TMA-staged pipeline (device sources, max_ctas == 0), the register path
(max_ctas > 0, used for mapped host memory), HND paged prefixes (per-head
bulk copies) and sources that are only element-aligned (direct fallback)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200 import _native

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _case(device, *, hnd: bool, misalign: bool, apc: int, heads=4, hd=128, bs=16, pool=512,
          tokens=2048, chunk=256, seed=0, neox=True, rotary_dim=None):
    rng = np.random.default_rng(seed)
    gen = torch.Generator(device=device).manual_seed(seed)
    if hnd:
        storage = torch.randn(2, pool, heads, bs, hd, generator=gen, device=device).to(torch.bfloat16)
        cache = storage.transpose(2, 3)  # [2, NB, BS, H, D] view of HND storage
    else:
        cache = torch.randn(2, pool, bs, heads, hd, generator=gen, device=device).to(torch.bfloat16)
    chunks = tokens // chunk
    hit_idx = np.sort(rng.choice(np.arange(apc // chunk + 1, chunks), size=4, replace=False))
    sources = rng.integers(0, 30000, size=4)
    row = heads * hd
    # packed hit buffer: per segment K plane then V plane; misaligned by one element if asked
    pad = 1 if misalign else 0
    hit = torch.randn(4 * 2 * chunk * row + pad + 8, generator=gen, device=device).to(torch.bfloat16)
    table = np.zeros(4, dtype=_native.SEGMENT_DTYPE)
    hosts = []
    base = hit.data_ptr() + 2 * pad
    for i in range(4):
        off = i * 2 * chunk * row
        table[i] = (base + off * 2, base + (off + chunk * row) * 2, row * 2, hd * 2,
                    int(sources[i]), int(hit_idx[i]) * chunk, chunk, 1)
        k = hit[pad + off: pad + off + chunk * row].reshape(chunk, heads, hd)
        v = hit[pad + off + chunk * row: pad + off + 2 * chunk * row].reshape(chunk, heads, hd)
        hosts.append(np.stack([_bits(k), _bits(v)]))
    blocks = rng.permutation(pool)[: tokens // bs]
    slots = (blocks[:, None] * bs + np.arange(bs)[None, :]).reshape(-1).astype(np.int64)
    alloc_end = int(hit_idx[-1]) * chunk + chunk
    token_segment = np.full(alloc_end, -1, dtype=np.int32)
    for i, c in enumerate(hit_idx):
        token_segment[int(c) * chunk:(int(c) + 1) * chunk] = i
    rd = rotary_dim or hd
    inv = 1.0 / (1e6 ** (np.arange(0, rd, 2, dtype=np.float64) / rd))
    freqs = np.arange(32768, dtype=np.float64)[:, None] * inv[None, :]
    cos_sin = oracle.f32_to_bf16(np.concatenate((np.cos(freqs), np.sin(freqs)), -1).astype(np.float32))
    return dict(cache=cache, hit=hit, table=table, hosts=hosts, slots=slots, alloc_end=alloc_end,
                token_segment=token_segment, cos_sin=cos_sin, sources=sources, hit_idx=hit_idx,
                heads=heads, hd=hd, bs=bs, chunk=chunk, apc=apc, hnd=hnd, neox=neox, rotary_dim=rd)


def _run(case, device, max_ctas: int, token_pad: int = 0):
    """``token_pad`` > 0 leaves a gap after every staging row (row-by-row kernel)."""
    c = case
    cache = c["cache"]
    heads, hd = c["heads"], c["hd"]
    rows = torch.empty(2, c["alloc_end"], heads * hd + token_pad, dtype=torch.bfloat16, device=device)
    out = rows[:, :, : heads * hd].unflatten(2, (heads, hd))
    slots = torch.from_numpy(c["slots"][: c["alloc_end"]]).to(device)
    token_segment = torch.from_numpy(c["token_segment"]).to(device)
    table = torch.from_numpy(c["table"].view(np.uint8)).to(device)
    cos_sin = torch.from_numpy(c["cos_sin"].view(np.int16)).view(torch.bfloat16).to(device)
    error = torch.zeros(1, dtype=torch.int32, device=device)
    esize = 2
    _native.call(
        "cb_blend_load_layer", out.data_ptr(), out.stride(0) * esize, out.stride(1) * esize, hd * esize,
        c["alloc_end"], c["apc"], cache[0].data_ptr(), cache[1].data_ptr(), cache.stride(1) * esize,
        cache.stride(2) * esize, cache.stride(3) * esize, cache.shape[1], c["bs"], slots.data_ptr(), heads,
        hd, 0, token_segment.data_ptr(), table.data_ptr(), 4, cos_sin.data_ptr(), cos_sin.shape[0],
        c["rotary_dim"], int(c["neox"]), max_ctas, error.data_ptr(), _native.stream_handle(),
    )
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    return _bits(out)


def _expected(case):
    c = case
    k_np = _bits(c["cache"][0])  # logical [NB, BS, H, D] content, whatever the storage order
    v_np = _bits(c["cache"][1])
    segs = [(int(c["sources"][i]), int(c["hit_idx"][i]) * c["chunk"], c["chunk"], c["hosts"][i])
            for i in range(4)]
    return oracle.blend_load(oracle.BF16, c["alloc_end"], c["apc"], k_np, v_np, c["slots"][: c["alloc_end"]],
                             c["bs"], segs, np.ones(4, dtype=np.int32), c["cos_sin"], c["hd"],
                             c["rotary_dim"], c["neox"])


@pytest.mark.parametrize("hnd", [False, True])
@pytest.mark.parametrize("misalign", [False, True])
@pytest.mark.parametrize("max_ctas", [0, 64])
def test_blend_load_paths_match_oracle(cuda, hnd, misalign, max_ctas):
    case = _case(cuda, hnd=hnd, misalign=misalign, apc=300, seed=int(hnd) * 2 + int(misalign))
    assert np.array_equal(_run(case, cuda, max_ctas), _expected(case))


@pytest.mark.parametrize("heads", [1, 2, 8, 16])
def test_blend_load_tma_tile_shapes(cuda, heads):
    # rows per 16 KiB tile from 64 (1 head) down to 4 (16 heads)
    case = _case(cuda, hnd=False, misalign=False, apc=0, heads=heads, seed=10 + heads)
    assert np.array_equal(_run(case, cuda, 0), _expected(case))


@pytest.mark.parametrize("heads,neox", [(1, True), (8, True), (8, False)])
def test_blend_load_strided_staging(cuda, heads, neox):
    """Staging rows with gaps between them: the row-by-row TMA kernel (no tile store)."""
    case = _case(cuda, hnd=False, misalign=False, apc=200, heads=heads, seed=30 + heads, neox=neox)
    assert np.array_equal(_run(case, cuda, 0, token_pad=64), _expected(case))


@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("token_pad", [0, 64])
def test_blend_load_partial_rotary(cuda, neox, token_pad):
    """rotary_dim 64 of head_size 128: the upper half of each head passes through."""
    case = _case(cuda, hnd=False, misalign=False, apc=100, heads=4, seed=40, neox=neox, rotary_dim=64)
    assert np.array_equal(_run(case, cuda, 0, token_pad=token_pad), _expected(case))


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("hnd,misalign", [(False, False), (True, False), (False, True)])
@pytest.mark.parametrize("neox,rotary_dim", [(True, 128), (False, 128), (True, 64)])
def test_blend_load_small_rows(cuda, heads, hnd, misalign, neox, rotary_dim):
    """Rows under 1 KiB (one or two heads per rank): the one-thread-per-item kernel."""
    case = _case(cuda, hnd=hnd, misalign=misalign, apc=300, heads=heads, neox=neox,
                 rotary_dim=rotary_dim, seed=50 + heads + 2 * hnd + 4 * misalign + 8 * neox)
    assert np.array_equal(_run(case, cuda, 0), _expected(case))


@pytest.mark.parametrize("max_ctas", [0, 64])
def test_blend_load_gptj_matches_oracle(cuda, max_ctas):
    case = _case(cuda, hnd=False, misalign=False, apc=100, seed=21, neox=False)
    assert np.array_equal(_run(case, cuda, max_ctas), _expected(case))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("contiguous", [True, False])
def test_relocate_key_random_vs_oracle(cuda, dtype, neox, contiguous):
    from cacheblend_b200.rope import relocate_key

    gen = torch.Generator(device=cuda).manual_seed(7)
    hd, heads, tokens, max_pos = 128, 8, 3000, 40960
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    freqs = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]

    class Rope:
        head_size = rotary_dim = hd
        is_neox_style = neox
        cos_sin_cache = torch.cat((freqs.cos(), freqs.sin()), -1).float().to(cuda)

    base = torch.randn(tokens, heads * hd + (0 if contiguous else 3), generator=gen, device=cuda).to(dtype)
    key = base[:, : heads * hd] if contiguous else base[:, 3:]  # 6-byte offset rows: scalar path
    old = torch.randint(0, max_pos, (tokens,), generator=gen, device=cuda)
    new = torch.randint(0, max_pos, (tokens,), generator=gen, device=cuda)
    out = relocate_key(Rope(), old, new, key)
    code = {torch.bfloat16: oracle.BF16, torch.float16: oracle.FP16, torch.float32: oracle.FP32}[dtype]
    table = Rope.cos_sin_cache.to(dtype).cpu()
    to_np = (lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)) if dtype == torch.bfloat16 \
        else (lambda t: t.contiguous().numpy())
    want = oracle.relocate(to_np(key.cpu()), to_np(table), old.cpu().numpy(), new.cpu().numpy(), hd, hd, neox,
                           code)
    assert np.array_equal(to_np(out.cpu()), want)
