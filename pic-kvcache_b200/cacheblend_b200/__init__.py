"""B200-native CacheBlend hot path behind the ``cacheblend_vllm`` connector API.

Hot-path ops (sm_100a kernels through the C ABI in include/cacheblend_b200.h):
``gather_paged_kv`` / ``scatter_paged_kv`` (K1), ``PagedBlendLoader`` with
``relocate_key`` (K2), ``kv_deviation`` / ``select_tokens`` (K3).  Host-side
mirrors of the reference types: ``CacheBlendConfig``, ``BlendPlan``,
``LocalPinnedCPUStore``, ``PipelineTracer``.
"""

from .config import CacheBlendConfig
from .kv_layout import gather_paged_kv, scatter_paged_kv
from .loader import PagedBlendLoader
from .rope import relocate_key, validate_rope_support
from .selection import kv_deviation, recompute_budget, select_tokens, sparse_q_masks
from .storage import LocalPinnedCPUStore
from .trace import PipelineTracer
from .types import BlendPlan, BlendSegment, SegmentId

__all__ = [
    "BlendPlan",
    "BlendSegment",
    "CacheBlendConfig",
    "LocalPinnedCPUStore",
    "PagedBlendLoader",
    "PipelineTracer",
    "SegmentId",
    "gather_paged_kv",
    "kv_deviation",
    "recompute_budget",
    "relocate_key",
    "scatter_paged_kv",
    "select_tokens",
    "sparse_q_masks",
    "validate_rope_support",
]
