"""The C-ABI library builds for sm_100a, loads without a GPU and exports every
entry point include/*.h declares, with the signatures the binding uses."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from cacheblend_b200 import _native

REPO = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for header in (REPO / "include").glob("*.h"):
        text = header.read_text()
        names.update(re.findall(r"CB_API\s+[\w\s\*]+?\b(cb_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = _native.load_library()
    declared = declared_symbols()
    assert declared, "no CB_API declarations found"
    for name in declared:
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr), name
    assert declared == set(_native.SIGNATURES), "binding table out of sync with the header"
    assert lib.cb_abi_version() == _native.ABI_VERSION


def test_argument_counts_match_header():
    text = "\n".join(h.read_text() for h in (REPO / "include").glob("*.h"))
    for name, (_, argtypes) in _native.SIGNATURES.items():
        match = re.search(rf"\b{name}\s*\(([^;]*?)\)\s*;", text, re.S)
        assert match, name
        params = [p for p in match.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(argtypes), name


def test_segment_struct_layout_matches_header():
    assert ctypes.sizeof(_native.CBSegment) == 48
    assert _native.SEGMENT_DTYPE.itemsize == 48


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _native.load_library()
    # negative sizes fail argument validation before any CUDA call
    rc = lib.cb_select_topk(None, None, 5, 9, None, 0, None)
    assert rc == _native.CB_ERR_INVALID
    assert b"n/k" in lib.cb_last_error()


def test_peer_exchange_buffer_layout_without_a_gpu():
    """cb_peer_select_buffer_size: receive rows [2][world][max_tokens rounded up to 4] of 8-byte
    entries (the low-latency words; the flag protocol's fp32 rows use half),
    then flags [8 ranks][8 cluster CTAs] and call counters [8] u32; world 1-8, at most one
    cluster's 344,064 scores.  Pure arithmetic: no CUDA call."""
    lib = _native.load_library()
    size = ctypes.c_int64(0)
    for world, tokens in ((1, 0), (2, 1), (2, 32768), (8, 32769), (8, 8 * 42 * 1024)):
        assert lib.cb_peer_select_buffer_size(world, tokens, ctypes.byref(size)) == _native.CB_OK
        capacity = (tokens + 3) // 4 * 4
        assert size.value == 2 * world * capacity * 8 + 9 * 8 * 4
    for world, tokens in ((0, 10), (9, 10), (2, -1), (2, 8 * 42 * 1024 + 1)):
        assert lib.cb_peer_select_buffer_size(world, tokens, ctypes.byref(size)) == _native.CB_ERR_INVALID
    assert lib.cb_peer_select_buffer_size(2, 10, None) == _native.CB_ERR_INVALID
    # a null buffer table is rejected before any device work
    assert lib.cb_select_topk_peer(None, None, 0, 0, None, 0, None, 0, 2, 0, 0, None, None, None) == \
        _native.CB_ERR_INVALID
    assert lib.cb_select_topk_peer(None, None, 0, 0, None, 0, None, 2, 2, 0, 0, None, None, None) == \
        _native.CB_ERR_INVALID  # rank outside the world
