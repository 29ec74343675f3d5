"""The collective policy: which backend carries which collective (CPU-only, no torch)."""

from .policy import (
    BACKENDS,
    GATHER_ALGORITHMS,
    MEASURED_TABLE,
    NVLINK_POLICY,
    PACK_BYTES,
    SUPPORTED_DTYPES,
    CollectivePolicy,
    MeasuredLimits,
    crossover_from_timings,
    derive_limits,
    load_measured,
    policy_for_profile,
    sweep_rows,
)

__all__ = ["BACKENDS", "GATHER_ALGORITHMS", "MEASURED_TABLE", "NVLINK_POLICY", "PACK_BYTES", "SUPPORTED_DTYPES",
           "CollectivePolicy", "MeasuredLimits", "crossover_from_timings", "derive_limits", "load_measured",
           "policy_for_profile", "sweep_rows"]
