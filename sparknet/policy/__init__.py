"""The collective policy: which backend carries which collective (CPU-only, no torch)."""

from .policy import (
    BACKENDS,
    GATHER_ALGORITHMS,
    NVLINK_POLICY,
    PACK_BYTES,
    SUPPORTED_DTYPES,
    CollectivePolicy,
    crossover_from_timings,
    policy_for_profile,
)

__all__ = ["BACKENDS", "GATHER_ALGORITHMS", "NVLINK_POLICY", "PACK_BYTES", "SUPPORTED_DTYPES", "CollectivePolicy",
           "crossover_from_timings", "policy_for_profile"]
