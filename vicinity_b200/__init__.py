"""B200-native IVF-PQ search engine with the interface of vicinity's IVF-PQ path.

The compute path is the CUDA library ``libvicinity_gpu.so`` (sm_100a),
reached through its C ABI (``include/vicinity_gpu.h``); this package is the
Python host binding, shaped like the reference's ``pyvicinity.IVFPQIndex``.
"""
from ._lib import VicinityError, device_count
from .ivf_pq import (
    MISSING_DISTANCE,
    MISSING_LABEL,
    FlatIndex,
    IVFPQFileSearcher,
    IVFPQIndex,
    current_generation,
    default_ivfpq_codebooks,
    flat_search_ip,
    nccl_unique_id,
    selftest_bounded_wait,
    shard_assign_lists,
    verify_generation,
)

__all__ = [
    "FlatIndex",
    "IVFPQFileSearcher",
    "IVFPQIndex",
    "current_generation",
    "MISSING_DISTANCE",
    "MISSING_LABEL",
    "VicinityError",
    "default_ivfpq_codebooks",
    "device_count",
    "flat_search_ip",
    "nccl_unique_id",
    "selftest_bounded_wait",
    "shard_assign_lists",
    "verify_generation",
]
