"""flashnext_b200 -- B200 (sm_100a) Flash-Next sparse-MoE decode path.

Host side of the C ABI in ``include/fnmoe.h``; the compute lives in
``libfnmoe.so`` (built in-tree from ``../csrc`` by ``../build.py``).  The
public surface mirrors the reference's op-level API for this path
(``models/flashnext/metal_runtime.py``, ``compiled.py``, ``adaptive_topk.py``,
``models/qwen27b/paged_kv.py``).  There is no CPU fallback.
"""
from __future__ import annotations

from .cuda_runtime import (  # noqa: F401
    BITS,
    GROUP_SIZE,
    MAX_EXPERTS,
    MAX_TOKENS,
    MAX_TOP_K,
    MAX_WIDTH,
    SUPPORTED_GROUP_SIZES,
    CudaCapabilities,
    MetalMoEExecutor,
    MoEExecutor,
    Q4G32Projection,
    probe_capabilities,
    weighted_combine,
)
from .expert_table import ExpertTable, RecordLayout, record_layout  # noqa: F401

__all__ = [
    "BITS", "GROUP_SIZE", "MAX_EXPERTS", "MAX_TOKENS", "MAX_TOP_K", "MAX_WIDTH",
    "SUPPORTED_GROUP_SIZES", "CudaCapabilities", "MetalMoEExecutor", "MoEExecutor",
    "Q4G32Projection", "probe_capabilities", "weighted_combine", "ExpertTable",
    "RecordLayout", "record_layout",
]
