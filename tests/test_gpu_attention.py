"""Blend attention on the tcgen05 tensor cores vs the reference's einsum path
(Qwen3BlendExecutor._attention, cacheblend_vllm/ascend.py:798-846) evaluated in
torch on the same device and dtype.

Default mode (the reference's order): the kernel rounds the normalized
probabilities to the element type T before P V, as the reference does, so
both sides round the same fp32 value p_j up to the last bits of exp / sum
(1e-6 relative) and sum p_j v_j in fp32 in different orders.  Each output is
then the same fp32 value up to accumulation order, rounded once on each side:

    |got - want| <= u (|got| + |want|) + 1e-6       (u = 2^-9 bf16, 2^-11 fp16)

for all but 1 % of the elements, and at least 98 % of the outputs are bit for
bit the reference's.  The exceptions: a probability whose fp32 value sits
within the last bits of exp / sum of a T midpoint rounds the other way on one
side (more often in fp16, whose grid is 8x finer), moving the output by up to
2u p_j |v_j|, which is large next to an output that cancels to near zero; and
a logit whose fp32 dot product lands within the accumulation-order difference
of a T midpoint rounds the other way.  Both stay within the flash-order bound
below.

Flash-order mode (derived bound): the kernel rounds p_j * L (the unnormalized
exp2 values, L a per-row factor) to T, sums, and divides by L at the end.
Each rounding is within u relative, so before the final rounding the two
results differ by at most 2u * sum_j p_j |v_j|, and the final rounding of each
side adds u |out| apiece:

    |got - want| <= 2u (P |V|) + u (|got| + |want|) + 1e-6

with P |V| computed from the reference's fp32 probabilities; logit flips as
above are allowed on at most 1e-4 of the elements (1e-3 in the peaked-logit
test) and within 4x.  The fused-logit mode compares with fp32 logits and its
own check.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from cacheblend_b200.attention import attention_workspace_bytes, blend_attention

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 2e-2
MEAN_TOL = 2e-3


def reference_attention(query, key, value, positions, scale, with_bound=False):
    """The reference formula, one KV head at a time (same roundings: the
    einsum output in the element type, scaled in the element type, masked with
    the type's minimum, softmax in fp32, probabilities cast back).  With
    ``with_bound`` also returns P |V| (fp32 probabilities times |v|)."""
    nq, hq, d = query.shape
    nk, hkv, _ = key.shape
    groups = hq // hkv
    masked = positions[:, None] < torch.arange(nk, device=query.device)[None, :]
    out = torch.empty_like(query)
    pv_abs = torch.empty(query.shape, dtype=torch.float32, device=query.device)
    # the reference's CPU einsum sums in fp32; cuBLAS may otherwise reduce split-K partial
    # sums in the element type
    flags = torch.backends.cuda.matmul
    saved = (flags.allow_bf16_reduced_precision_reduction, flags.allow_fp16_reduced_precision_reduction)
    flags.allow_bf16_reduced_precision_reduction = False
    flags.allow_fp16_reduced_precision_reduction = False
    try:
        _reference_heads(query, key, value, scale, masked, groups, out, pv_abs, with_bound)
    finally:
        flags.allow_bf16_reduced_precision_reduction, flags.allow_fp16_reduced_precision_reduction = saved
    return (out, pv_abs) if with_bound else out


def _reference_heads(query, key, value, scale, masked, groups, out, pv_abs, with_bound):
    for h in range(key.shape[1]):
        q = query[:, h * groups:(h + 1) * groups]              # [nq, g, d]
        weights = torch.einsum("qgd,kd->gqk", q, key[:, h]) * scale
        weights = weights.masked_fill(masked[None], torch.finfo(weights.dtype).min)
        p32 = torch.softmax(weights.float(), dim=-1)
        out[:, h * groups:(h + 1) * groups] = torch.einsum("gqk,kd->qgd", p32.to(query.dtype), value[:, h])
        if with_bound:
            pv_abs[:, h * groups:(h + 1) * groups] = torch.einsum("gqk,kd->qgd", p32, value[:, h].float().abs())


def _unit_roundoff(dtype) -> float:
    return 2.0 ** -9 if dtype == torch.bfloat16 else 2.0 ** -11


def _check_bound(got, want, pv_abs, max_bad_fraction=1e-4):
    """The derived per-element bound (module docstring)."""
    u = _unit_roundoff(got.dtype)
    g, w = got.float(), want.float()
    diff = (g - w).abs()
    bound = 2 * u * pv_abs + u * (g.abs() + w.abs()) + 1e-6
    bad = int((diff > bound).sum())
    assert bad <= max_bad_fraction * diff.numel(), (
        f"{bad} of {diff.numel()} elements beyond the derived bound, worst ratio "
        f"{float((diff / bound).max()):.3g}")
    assert bool((diff <= 4 * bound).all()), f"worst ratio {float((diff / bound).max()):.3g}"


def _check_order(got, want, pv_abs, max_bad_fraction=1e-4, min_equal=0.98, max_off_fraction=1e-2):
    """The reference-order mode: one rounding of the same value on each side
    (module docstring), within the flash-order bound everywhere."""
    u = _unit_roundoff(got.dtype)
    g, w = got.float(), want.float()
    diff = (g - w).abs()
    equal = float((diff == 0).float().mean())
    assert equal >= min_equal, f"only {equal:.4f} of the outputs equal the reference's"
    tight = u * (g.abs() + w.abs()) + 1e-6
    off = int((diff > tight).sum())
    assert off <= max_off_fraction * diff.numel(), (
        f"{off} of {diff.numel()} elements beyond one rounding, worst ratio {float((diff / tight).max()):.3g}")
    _check_bound(got, want, pv_abs, max_bad_fraction=max_bad_fraction)


def _check_reference(got, query, key, value, positions, scale, max_bad_fraction=1e-4, mode="reference"):
    want, pv_abs = reference_attention(query, key, value, positions, scale, with_bound=True)
    if mode == "reference":
        _check_order(got, want, pv_abs, max_bad_fraction=max_bad_fraction)
    else:
        _check_bound(got, want, pv_abs, max_bad_fraction)


def _check(got, want, max_bad_fraction=0.0):
    diff = (got.float() - want.float()).abs()
    bound = ATOL + RTOL * want.float().abs()
    bad = int((diff > bound).sum())
    assert bad <= max_bad_fraction * diff.numel(), (
        f"{bad} elements out of tolerance, max diff {float(diff.max()):.4g}")
    assert float(diff.mean()) < MEAN_TOL


def _inputs(cuda, nq, nk, hq, hkv, dtype, seed, pruned=True):
    gen = torch.Generator(device=cuda).manual_seed(seed)
    if pruned:
        # computed rows: a sorted random subset of positions that always
        # includes the last one (the suffix of a blend request)
        pick = torch.randperm(nk - 1, generator=gen, device=cuda)[: nq - 1]
        positions = torch.cat([pick.sort().values, torch.tensor([nk - 1], device=cuda)])
    else:
        positions = torch.arange(nk - nq, nk, device=cuda)
    query = torch.randn(nq, hq, 128, generator=gen, device=cuda).to(dtype)
    key = torch.randn(nk, hkv, 128, generator=gen, device=cuda).to(dtype)
    value = torch.randn(nk, hkv, 128, generator=gen, device=cuda).to(dtype)
    return query, key, value, positions


def _to_device(bits, code, device):
    dtype = torch.bfloat16 if code == 0 else torch.float16
    return torch.from_numpy(bits.view(np.int16)).view(dtype).to(device)


@pytest.mark.parametrize("case", range(3))
def test_attention_golden(attention_golden, cuda, case):
    """Against the reference's own outputs (tests/golden/attention.npz)."""
    tag = f"att_{case}"
    code = int(attention_golden[f"{tag}_meta"][0])
    q, k, v = (_to_device(attention_golden[f"{tag}_{n}"], code, cuda) for n in ("query", "key", "value"))
    positions = torch.from_numpy(attention_golden[f"{tag}_positions"]).to(cuda)
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = blend_attention(q, k, v, positions, float(attention_golden[f"{tag}_scale"][0]), device_error=error)
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    _, pv_abs = reference_attention(q, k, v, positions, float(attention_golden[f"{tag}_scale"][0]),
                                    with_bound=True)
    _check_order(got, _to_device(attention_golden[f"{tag}_out"], code, cuda), pv_abs)


def test_attention_vs_oracle(cuda):
    """Against the CPU oracle on a seeded case with ragged tiles."""
    query, key, value, positions = _inputs(cuda, 150, 420, 8, 2, torch.bfloat16, 17)
    got = blend_attention(query, key, value, positions, 0.09)
    as_np = lambda t: t.float().cpu().numpy()
    want = oracle.blend_attention(as_np(query), as_np(key), as_np(value), positions.cpu().numpy(), 0.09,
                                  oracle.BF16)
    _, pv_abs = reference_attention(query, key, value, positions, 0.09, with_bound=True)
    _check_order(got, torch.from_numpy(want).to(cuda).to(torch.bfloat16), pv_abs)


@pytest.mark.parametrize(
    "nq,nk,hq,hkv,dtype,pruned",
    [
        (300, 300, 32, 8, torch.bfloat16, False),   # prefill: every position computed
        (160, 1000, 16, 2, torch.bfloat16, True),   # pruned rows, ragged key count
        (77, 77, 8, 8, torch.float16, False),       # one query per head (groups 1), fp16
        (250, 2100, 64, 4, torch.bfloat16, True),   # groups 16
        (1, 129, 32, 8, torch.bfloat16, True),      # single query, keys one past a tile
        (1229, 8192, 32, 8, torch.bfloat16, True),  # Qwen3-8B heads, 15% of 8k rows
    ],
)
@pytest.mark.parametrize("mode", ["reference", "flash"])
def test_attention_vs_reference(cuda, nq, nk, hq, hkv, dtype, pruned, mode):
    query, key, value, positions = _inputs(cuda, nq, nk, hq, hkv, dtype, nq * 7 + nk, pruned)
    scale = 128 ** -0.5
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = blend_attention(query, key, value, positions, scale, device_error=error, exact_rounding=mode)
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    _check_reference(got, query, key, value, positions, scale, mode=mode)


@pytest.mark.parametrize("mode", ["reference", "flash"])
def test_attention_peaked_logits(cuda, mode):
    """Large logits: row maxima grow across key tiles by more than the lazy
    rescale threshold, so the output accumulator is rescaled in TMEM.  Here a
    logit's element-type rounding is a large step (1/8 at 30), and the two
    fp32 accumulation orders can round a logit near a midpoint differently;
    when that logit dominates its row the output moves by more than the
    tolerance, so up to 1e-3 of the elements may differ by more."""
    query, key, value, positions = _inputs(cuda, 200, 1500, 16, 4, torch.bfloat16, 11)
    # keys grow in magnitude with position so later tiles raise each row's max
    key = (key.float() * torch.linspace(0.5, 3.0, key.shape[0], device=cuda)[:, None, None]).to(key.dtype)
    scale = 0.5
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = blend_attention(query, key, value, positions, scale, device_error=error, exact_rounding=mode)
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    _check_reference(got, query, key, value, positions, scale, max_bad_fraction=1e-3, mode=mode)


def test_attention_strided_views(cuda):
    """Query / key / value as column slices of one packed QKV projection (the
    executor's layout), output into a wider buffer through a view."""
    nq, nk, hq, hkv = 180, 640, 32, 8
    gen = torch.Generator(device=cuda).manual_seed(5)
    width = (hq + 2 * hkv) * 128
    qkv = torch.randn(nk, width, generator=gen, device=cuda).to(torch.bfloat16)
    key = qkv[:, hq * 128:(hq + hkv) * 128].view(nk, hkv, 128)
    value = qkv[:, (hq + hkv) * 128:].view(nk, hkv, 128)
    positions = torch.randperm(nk, generator=gen, device=cuda)[:nq].sort().values
    query = qkv[positions, : hq * 128].view(nq, hq, 128)
    query = torch.empty(nq, width, dtype=torch.bfloat16, device=cuda)[:, : hq * 128].copy_(
        query.reshape(nq, -1)).view(nq, hq, 128)
    assert query.stride(0) == width
    got = blend_attention(query, key, value, positions, 128 ** -0.5)
    _check_reference(got, query, key, value, positions, 128 ** -0.5)


def test_attention_workspace_reuse(cuda):
    """A caller-owned workspace sized for the largest shape serves smaller calls."""
    query, key, value, positions = _inputs(cuda, 400, 3000, 32, 8, torch.bfloat16, 3)
    need = attention_workspace_bytes(400, 3000, 32, 8, 128, torch.bfloat16)
    workspace = torch.empty(need, dtype=torch.uint8, device=cuda)
    for nq, nk in ((400, 3000), (90, 700)):
        q = query[:nq]
        pos = torch.clamp(positions[:nq], max=nk - 1)
        got = blend_attention(q, key[:nk], value[:nk], pos, 0.1, workspace=workspace)
        _check_reference(got, q, key[:nk], value[:nk], pos, 0.1)


def test_attention_rejects_unsupported(cuda):
    q = torch.zeros(4, 8, 64, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(4, 8, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(NotImplementedError):
        blend_attention(q, k, k, torch.arange(4, device=cuda), 1.0)
    q = torch.zeros(4, 8, 128, dtype=torch.float32, device=cuda)
    with pytest.raises(NotImplementedError):
        blend_attention(q, q, q, torch.arange(4, device=cuda), 1.0)


@pytest.mark.parametrize(
    "nq,nk,hq,hkv,positions",
    [
        (1, 1, 8, 8, "zero"),        # a single key
        (40, 300, 16, 4, "zero"),    # every query at position 0: one key each
        (64, 640, 32, 1, "dup"),     # 32 query heads on one KV head; repeated positions
        (97, 127, 8, 2, "last"),     # keys one short of a tile
        (97, 128, 8, 2, "last"),     # keys exactly one tile
        (300, 256, 8, 8, "dup"),     # groups 1, 300 rows: pairs of 128-row tiles, padding
    ],
)
def test_attention_edge_shapes(cuda, nq, nk, hq, hkv, positions):
    gen = torch.Generator(device=cuda).manual_seed(nq + nk)
    if positions == "zero":
        pos = torch.zeros(nq, dtype=torch.long, device=cuda)
    elif positions == "last":
        pos = torch.full((nq,), nk - 1, dtype=torch.long, device=cuda)
    else:
        pos = torch.randint(0, nk, (nq,), generator=gen, device=cuda).sort().values
    query = torch.randn(nq, hq, 128, generator=gen, device=cuda).to(torch.bfloat16)
    key = torch.randn(nk, hkv, 128, generator=gen, device=cuda).to(torch.bfloat16)
    value = torch.randn(nk, hkv, 128, generator=gen, device=cuda).to(torch.bfloat16)
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = blend_attention(query, key, value, pos, 128 ** -0.5, device_error=error)
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    _check_reference(got, query, key, value, pos, 128 ** -0.5)
    if positions == "zero":  # one visible key: the output is that key's value row
        assert torch.equal(got, value[0][None].repeat_interleave(hq // hkv, dim=1).expand_as(got))


def test_attention_rejects_misaligned_rows(cuda):
    base = torch.zeros(8 * 129 * 128 + 8, dtype=torch.bfloat16, device=cuda)
    # rows 129 heads apart would be fine; an odd element offset breaks 16-byte alignment
    key = base[1 : 1 + 8 * 2 * 128].view(8, 2, 128)
    query = torch.zeros(4, 2, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(NotImplementedError):
        blend_attention(query, key, key, torch.arange(4, device=cuda), 1.0)


def fused_reference(query, key, value, positions, scale):
    """The reference's fused-kernel semantics (ascend.py:814-830): fp32 logits times
    the scale, fp32 softmax over keys <= position, output in the element type.
    Returns (out, P |V|) for the derived bound."""
    groups = query.shape[1] // key.shape[1]
    masked = positions[:, None] < torch.arange(key.shape[0], device=query.device)[None, :]
    out = torch.empty_like(query)
    pv_abs = torch.empty(query.shape, dtype=torch.float32, device=query.device)
    for h in range(key.shape[1]):
        q = query[:, h * groups:(h + 1) * groups].float()
        w = torch.einsum("qgd,kd->gqk", q, key[:, h].float()) * scale
        w = w.masked_fill(masked[None], float("-inf"))
        p = torch.softmax(w, dim=-1)
        out[:, h * groups:(h + 1) * groups] = torch.einsum("gqk,kd->qgd", p, value[:, h].float()).to(query.dtype)
        pv_abs[:, h * groups:(h + 1) * groups] = torch.einsum("gqk,kd->qgd", p, value[:, h].float().abs())
    return out, pv_abs


@pytest.mark.parametrize("nq,nk,hq,hkv,dtype", [(300, 1000, 32, 8, torch.bfloat16), (77, 77, 8, 8, torch.float16),
                                                (1229, 8192, 32, 8, torch.bfloat16)])
def test_attention_fused_logits(cuda, nq, nk, hq, hkv, dtype):
    query, key, value, positions = _inputs(cuda, nq, nk, hq, hkv, dtype, nq + 3 * nk)
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = blend_attention(query, key, value, positions, 128 ** -0.5, device_error=error, exact_rounding=False)
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    _check_bound(got, *fused_reference(query, key, value, positions, 128 ** -0.5))
    # the two modes differ by the logit roundings (up to u |logit| each): a few ulps apart
    _check(got, blend_attention(query, key, value, positions, 128 ** -0.5))


def test_attention_fused_logits_rejects_nonpositive_scale(cuda):
    q = torch.zeros(4, 8, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(4, 8, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        blend_attention(q, k, k, torch.arange(4, device=cuda), -1.0, exact_rounding=False)


def test_attention_positions_past_the_last_key(cuda):
    """A query position at or past the last staging row sees every key, as the
    reference's mask over the existing keys lets it."""
    query, key, value, _ = _inputs(cuda, 40, 300, 16, 4, torch.bfloat16, 77)
    pos = torch.tensor([299, 300, 5000] + list(range(100, 137)), device=cuda)
    got = blend_attention(query, key, value, pos, 128 ** -0.5)
    _check_reference(got, query, key, value, pos, 128 ** -0.5)


def test_attention_rejects_unknown_mode(cuda):
    q = torch.zeros(4, 8, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        blend_attention(q, q, q, torch.arange(4, device=cuda), 1.0, exact_rounding="exact")
