"""The FMA-pipe exp2 of the Sparse-Q epilogue (exp2_poly in
pic-kvcache_b200/csrc/sparse_q.cu), restated in numpy bit for bit: the
constants compiled into the kernel are the Remez fit of
pic-kvcache_b200/csrc/exp2_poly_fit.py, and the whole evaluation (clamp,
1.5*2^23 rounding split, Horner polynomial, exponent insertion) stays within
7.5e-5 relative of 2^y for y >= -125, and non-negative below 2^-124 for
smaller y (where the MUFU ex2.ftz returns 0 or a value below 2^-125).  CPU only."""

from __future__ import annotations

import importlib.util
import re
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]
CSRC = REPO / "pic-kvcache_b200" / "csrc"
BOUND = 7.5e-5


def _fit_module():
    spec = importlib.util.spec_from_file_location("exp2_poly_fit", CSRC / "exp2_poly_fit.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _kernel_constants() -> dict[str, np.float32]:
    text = (CSRC / "sparse_q.cu").read_text()
    found = dict(re.findall(r"constexpr float (kExp2\w+) = ([0-9.e+-]+)f;", text))
    return {name: np.float32(float(value)) for name, value in found.items()}


def _f32(x):
    return np.asarray(x, dtype=np.float32)


def _fma(a: np.ndarray, b, d) -> np.ndarray:
    """fp32 fused multiply-add: exact product and sum, one rounding."""
    return _f32(np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(d, np.float64))


def exp2_poly_reference(y: np.ndarray, c: dict[str, np.float32]) -> np.ndarray:
    """exp2_poly, step by step in fp32 (every add / fma rounded once, like the kernel)."""
    y = np.maximum(_f32(y), np.float32(-126.0))
    t = _f32(y + c["kExp2Round"])
    j = _f32(t - c["kExp2Round"])
    f = _f32(y.astype(np.float64) - j.astype(np.float64))
    p = _fma(f, c["kExp2C3"], c["kExp2C2"])
    p = _fma(p, f, c["kExp2C1"])
    p = _fma(p, f, c["kExp2C0"])
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def test_kernel_constants_are_the_remez_fit():
    fit = _fit_module()
    c = _kernel_constants()
    assert c["kExp2Round"] == np.float32(1.5 * 2**23)
    text = (CSRC / "sparse_q.cu").read_text()
    assert "fmaxf(y.x, -126.0f)" in text and "fmaxf(y.y, -126.0f)" in text  # the clamp restated below
    coeffs = fit.remez(3).astype(np.float32)
    kernel = np.array([c["kExp2C0"], c["kExp2C1"], c["kExp2C2"], c["kExp2C3"]], dtype=np.float32)
    np.testing.assert_allclose(kernel, coeffs, rtol=1e-6, atol=0)
    assert fit.fp32_max_relative_error(kernel) < BOUND


def test_exp2_poly_error_bound_over_the_score_range():
    c = _kernel_constants()
    y = np.concatenate([np.linspace(-125.0, 0.0, 1_000_003), -np.logspace(-8, 0, 10_001),
                        [0.0, -0.5, -1.5, -124.5, -125.0]]).astype(np.float32)
    got = exp2_poly_reference(y, c).astype(np.float64)
    want = np.exp2(y.astype(np.float64))
    assert np.max(np.abs(got / want - 1.0)) < BOUND
    # at the bottom of the range: tiny and non-negative whatever the input
    deep = np.concatenate([np.linspace(-1e4, -125.0, 100_001), [-np.inf, -3e38]]).astype(np.float32)
    small = exp2_poly_reference(deep, c)
    assert np.all(small >= 0) and np.all(small < 2.0**-124)
