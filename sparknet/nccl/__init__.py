"""NCCL control profiles for NVSwitch boxes (stock NCCL; no patch series is needed)."""

from .patchset import export as export_patches, patch_directory, series
from .profiles import (
    COMMON_ENV,
    COMMON_IB_ENV,
    PATCH_CONTROLS,
    PROFILES,
    REFERENCE_IB_ENV,
    environment,
    problems,
    profile,
    profile_problems,
    profiles_for,
    required_patches,
    size_bytes,
)

__all__ = ["COMMON_ENV", "COMMON_IB_ENV", "PATCH_CONTROLS", "PROFILES", "REFERENCE_IB_ENV", "environment", "export_patches",
           "patch_directory", "problems", "profile", "profile_problems", "profiles_for", "required_patches",
           "series", "size_bytes"]
