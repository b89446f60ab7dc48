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
