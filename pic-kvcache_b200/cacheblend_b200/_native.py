"""ctypes binding of ``libcacheblend_b200.so`` (the sm_100a C ABI in include/cacheblend_b200.h).

The library is built in-tree by ``pic-kvcache_b200/build.py``.  There is no
fallback: every hot-path op raises if the library is missing or if it is
handed CPU tensors.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import numpy as np
import torch

# CACHEBLEND_B200_LIB points at another build of the same ABI (e.g. a debug
# or tuning build); by default the library built in-tree next to this file.
LIB_PATH = Path(
    os.environ.get("CACHEBLEND_B200_LIB")
    or Path(__file__).resolve().parent / "_lib" / "libcacheblend_b200.so"
)
ABI_VERSION = 6

CB_OK = 0
CB_ERR_INVALID = -1
CB_ERR_UNSUPPORTED = -2
CB_ERR_CUDA = -3

DTYPE_CODES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_ptr = ctypes.c_void_p


class CBSegment(ctypes.Structure):
    """Mirror of ``cb_segment_t``."""

    _fields_ = [
        ("k_src", ctypes.c_uint64),
        ("v_src", ctypes.c_uint64),
        ("src_token_stride", ctypes.c_int64),
        ("src_head_stride", ctypes.c_int64),
        ("source_start", ctypes.c_int32),
        ("target_start", ctypes.c_int32),
        ("length", ctypes.c_int32),
        ("rotate", ctypes.c_int32),
    ]


# numpy view of the same struct, used to build descriptor tables in bulk.
SEGMENT_DTYPE = np.dtype(
    [
        ("k_src", np.uint64),
        ("v_src", np.uint64),
        ("src_token_stride", np.int64),
        ("src_head_stride", np.int64),
        ("source_start", np.int32),
        ("target_start", np.int32),
        ("length", np.int32),
        ("rotate", np.int32),
    ]
)
assert SEGMENT_DTYPE.itemsize == ctypes.sizeof(CBSegment) == 48

# name -> (restype, argtypes); must match include/cacheblend_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "cb_abi_version": (_i32, []),
    "cb_last_error": (ctypes.c_char_p, []),
    "cb_paged_gather": (
        _i32,
        [_ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _i64,
         _ptr, _i64, _i64, _i64, _i64, _i64, _ptr],
    ),
    "cb_paged_scatter": (
        _i32,
        [_ptr, _i64, _i64, _i64, _i64, _i64, _ptr, _ptr, _i64, _i64, _i64,
         _i64, _i64, _i64, _i64, _ptr, _i64, _ptr],
    ),
    "cb_paged_copy_error": (_i32, [_ptr, _ptr, _i32]),
    "cb_sorted_overlap": (_i32, [_ptr, _i64, _ptr, _i64, _ptr, _ptr]),
    "cb_copy_rows_d2h": (_i32, [_ptr, _i64, _ptr, _i64, _i64, _i64, _ptr]),
    "cb_window_hashes": (_i32, [_ptr, _i64, _i64, _ptr]),
    "cb_wait_selftest": (_i32, [_ptr, _ptr]),
    "cb_hash_candidates": (_i32, [_ptr, _i64, _ptr, _i64, _ptr, _i64, _ptr]),
    "cb_relocate_key": (
        _i32,
        [_ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _ptr, _i64,
         _ptr, _ptr, _ptr],
    ),
    "cb_blend_load_layer": (
        _i32,
        [_ptr, _i64, _i64, _i64, _i64, _i64, _ptr, _ptr, _i64, _i64, _i64, _i64,
         _i64, _ptr, _i64, _i64, _i32, _ptr, _ptr, _i64, _ptr, _i64, _i64, _i32,
         _i64, _ptr, _ptr],
    ),
    "cb_kv_deviation": (
        _i32,
        [_ptr, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i32, _ptr, _ptr],
    ),
    "cb_select_topk": (_i32, [_ptr, _ptr, _i64, _i64, _ptr, _i64, _ptr]),
    "cb_peer_select_buffer_size": (_i32, [_i32, _i64, _ptr]),
    "cb_peer_buffer_create": (_i32, [_i32, _i64, _ptr, _ptr]),
    "cb_peer_buffer_open": (_i32, [_i32, _ptr, _ptr]),
    "cb_peer_buffer_close": (_i32, [_i32, _ptr]),
    "cb_peer_buffer_destroy": (_i32, [_i32, _ptr]),
    "cb_peer_buffer_reset": (_i32, [_ptr, _i32, _i64, _ptr]),
    "cb_select_topk_peer": (
        _i32, [_ptr, _ptr, _i64, _i64, _ptr, _i64, _ptr, _i32, _i32, _i64, _i32, _ptr, _ptr, _ptr]),
    "cb_select_topk_peer_all_ranks": (
        _i32, [_ptr, _ptr, _i64, _i64, _ptr, _i64, _ptr, _i32, _i64, _i32, _ptr, _ptr, _ptr]),
    "cb_kv_deviation_select_workspace_size": (_i32, [_ptr]),
    "cb_kv_deviation_select": (
        _i32,
        [_ptr, _i64, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i32, _ptr, _i64, _ptr, _ptr, _i64,
         _ptr, _i64, _ptr],
    ),
    "cb_blend_attention_workspace_size": (_i32, [_i64, _i64, _i64, _i64, _i64, _i32, _ptr]),
    "cb_blend_attention": (
        _i32,
        [_ptr, _i64, _ptr, _i64, _ptr, _i64, _i64, _i64, _i64, _i64, _i32, _ptr, _i64,
         ctypes.c_float, _i32, _ptr, _i64, _ptr, _i64, _ptr, _ptr],
    ),
    "cb_sparse_q_workspace_size": (_i32, [_i64, _i64, _i64, _i64, _i32, _ptr]),
    "cb_sparse_q_scores": (
        _i32,
        [_ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64, _i64, _i32, _ptr, _ptr, _i64,
         ctypes.c_float, _ptr, _ptr, _i64, _ptr, _ptr],
    ),
    "cb_sparse_q_scores_static": (
        _i32,
        [_ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64, _i64, _i32, _ptr, _ptr, _i64,
         ctypes.c_float, _ptr, _ptr, _ptr],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load_library() -> ctypes.CDLL:
    """Load and type the shared library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"CacheBlend B200 library not found at {LIB_PATH}; "
                "build it with `python pic-kvcache_b200/build.py`"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.cb_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"libcacheblend_b200 ABI {version} != expected {ABI_VERSION}")
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Invoke a C-ABI entry point and translate its status into an exception."""
    lib = load_library()
    rc = getattr(lib, name)(*args)
    if rc != CB_OK:
        message = lib.cb_last_error().decode(errors="replace")
        if rc == CB_ERR_INVALID:
            raise ValueError(f"{name}: {message}")
        if rc == CB_ERR_UNSUPPORTED:
            raise NotImplementedError(f"{name}: {message}")
        raise RuntimeError(f"{name}: {message}")


def require_cuda(*tensors: torch.Tensor) -> None:
    for tensor in tensors:
        if tensor.device.type != "cuda":
            raise RuntimeError(
                "CacheBlend B200 kernels operate on CUDA tensors only "
                f"(got a {tensor.device.type} tensor); there is no CPU fallback"
            )


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError as error:
        raise NotImplementedError(f"unsupported element type {dtype}") from error


def stream_handle(stream: torch.cuda.Stream | None = None) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)
