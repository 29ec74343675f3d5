"""Named transport profiles for one NVSwitch box: the NCCL settings and collective
limits measured together (replaces the reference's Spark profiles,
``sparknet/nccl/profiles.py:74-268``).

A value of ``None`` means "omit the variable, use the library default", never zero.
On B200 NCCL runs unpatched over NVLink/NVSwitch; it is the baseline and the
large-message backend, so the profiles are mostly "stock" plus the sparknet limits.
``ib-forced-nccl-only`` reproduces the reference's NCCL-only control environment
verbatim (NCCL forced onto IB/RoCE with P2P, SHM and NVLS disabled), which is what
the reference's own NCCL-only profile measures.
"""

from __future__ import annotations

import re
from typing import Any

# The reference's shared fabric policy for its NCCL-only control (IB/RoCE forced).
REFERENCE_IB_ENV = {
    "NCCL_NET": "IB",
    "NCCL_NET_PLUGIN": "none",
    "NCCL_IB_DISABLE": "0",
    "NCCL_IB_MERGE_NICS": "1",
    "NCCL_IB_SUBNET_AWARE_ROUTING": "1",
    "NCCL_IB_ADDR_FAMILY": "AF_INET",
    "NCCL_IB_ROCE_VERSION_NUM": "2",
    "NCCL_CROSS_NIC": "1",
    "NCCL_IGNORE_CPU_AFFINITY": "1",
    "NCCL_P2P_DISABLE": "1",
    "NCCL_SHM_DISABLE": "1",
    "NCCL_NVLS_ENABLE": "0",
    "NCCL_DEBUG": "WARN",
    "NCCL_DEBUG_SUBSYS": "INIT",
    "TORCH_NCCL_ASYNC_ERROR_HANDLING": "1",
}
COMMON_IB_ENV = REFERENCE_IB_ENV  # the reference's name for the same environment
# Every NVLink profile shares these: asynchronous error handling and quiet logs.
COMMON_ENV = {
    "NCCL_DEBUG": "WARN",
    "TORCH_NCCL_ASYNC_ERROR_HANDLING": "1",
}
# No NCCL patches are needed on B200: the reference's series fixes an AArch64 fence
# and tunes switchless RoCE rings, neither of which exists on an NVSwitch box.
PATCH_CONTROLS: dict[str, tuple[str, ...]] = {}

_LIMITS = {
    "ALLREDUCE_CAPACITY_BYTES": "8388608",
    "ALLREDUCE_DISPATCH_MAX_BYTES": "2097152",
    "ALLGATHER_MAX_BYTES": "16777216",
    "TIMEOUT_MS": "10000",
}
_NO_LIMITS = {key: None for key in _LIMITS}


def _measured_limits(world: int) -> dict[str, str]:
    """The limits of a profile pinned to one world size: the all-reduce dispatch ceiling
    measured for it (``sparknet/policy/measured_b200.json``), with the registered capacity
    raised to hold it; the general limits where nothing was measured."""
    from sparknet.policy.policy import default_dispatch_bytes

    limits = dict(_LIMITS)
    dispatch = default_dispatch_bytes(world)
    limits["ALLREDUCE_DISPATCH_MAX_BYTES"] = str(dispatch)
    limits["ALLREDUCE_CAPACITY_BYTES"] = str(max(int(_LIMITS["ALLREDUCE_CAPACITY_BYTES"]), dispatch))
    return limits
_WORLDS = (1, 2, 4, 8)

PROFILES: dict[str, dict[str, Any]] = {
    "nvlink": {
        "transport": "nvlink",
        "node_counts": _WORLDS,
        "status": "product: sparknet one-shot/two-shot kernels up to the dispatch limit, stock NCCL above it",
        "nccl": {"NCCL_NVLS_ENABLE": None, "NCCL_P2P_LEVEL": None, "NCCL_ALGO": None, "NCCL_PROTO": None},
        "limits": dict(_LIMITS),
        "evidence": "bench.py and probe receipts on 8x B200 (profiles/ summaries)",
    },
    "nvlink-8": {
        "transport": "nvlink",
        "node_counts": (8,),
        "status": "product on a full box: as nvlink, pinned to tensor-parallel size 8 (every GPU of an HGX B200), "
                  "with the all-reduce dispatch ceiling measured at 8 GPUs (the NVLink kernels beat NCCL up to it)",
        "nccl": {"NCCL_NVLS_ENABLE": None, "NCCL_P2P_LEVEL": None, "NCCL_ALGO": None, "NCCL_PROTO": None},
        "limits": _measured_limits(8),
        "evidence": "bench.py --gpus 8, the decode benchmark and the 8-GPU probe sweep on 8x B200",
    },
    "nvlink-nvls": {
        "transport": "nvlink-nvls",
        "node_counts": (2, 4, 8),
        "status": "opt-in: as nvlink, plus NVLS multicast kernels for large messages (sums not in rank order)",
        "nccl": {"NCCL_NVLS_ENABLE": "1"},
        "limits": dict(_LIMITS),
        "evidence": "bench.py --algorithm nvls receipts on 8x B200",
    },
    "nvlink-nccl-only": {
        "transport": "nccl-nvlink",
        "node_counts": _WORLDS,
        "status": "control arm B: every collective on stock NCCL over NVLink/NVSwitch (NVLS as NCCL chooses)",
        "nccl": {"NCCL_NVLS_ENABLE": None},
        "limits": dict(_NO_LIMITS),
        "evidence": "bench.py --impl reference receipts (the reference's NCCL-only arm)",
    },
    "ib-forced-nccl-only": {
        "transport": "nccl-nvlink",
        "node_counts": _WORLDS,
        "status": "control arm A: the reference's direct-nccl-only environment verbatim (IB forced, P2P/SHM/NVLS "
                  "off); initialises only where an IB/RoCE device exists",
        "nccl": dict(REFERENCE_IB_ENV),
        "limits": dict(_NO_LIMITS),
        "evidence": "bench.py --impl reference --reference-env profile",
    },
}


def size_bytes(value: str) -> int:
    """``2MB`` -> bytes; KB/MB/GB are binary units."""
    match = re.fullmatch(r"([1-9][0-9]*)(B|KB|MB|GB)?", str(value))
    if not match:
        raise ValueError(f"invalid positive byte size: {value!r}")
    return int(match[1]) * {None: 1, "B": 1, "KB": 1024, "MB": 1024 ** 2, "GB": 1024 ** 3}[match[2]]


def profile(name: str) -> dict[str, Any]:
    """The named NCCL control profile (ValueError naming the known ones otherwise)."""
    try:
        return PROFILES[name]
    except KeyError:
        raise ValueError(f"unknown transport profile {name!r}; choose {', '.join(PROFILES)}") from None


def profiles_for(transport: str, world: int) -> list[str]:
    """The profiles that apply to ``transport`` at ``world`` GPUs."""
    return [n for n, e in PROFILES.items() if e["transport"] == transport and world in e["node_counts"]]


def profile_problems(name: str, transport: str, world: int) -> list[str]:
    """Why profile ``name`` does not fit ``transport`` at ``world`` GPUs (empty when it does)."""
    entry = profile(name)
    errors = []
    if entry["transport"] != transport:
        errors.append(f"profile {name} is for transport {entry['transport']}, not {transport}")
    if world not in entry["node_counts"]:
        errors.append(f"profile {name} applies to {', '.join(map(str, entry['node_counts']))} GPUs, not {world}")
    return errors


def environment(name: str) -> dict[str, str]:
    """The rank-invariant environment of a profile (per-node keys come from ``sparknet.topology``)."""
    entry = profile(name)
    env = dict(COMMON_ENV)
    for key, value in entry["nccl"].items():
        if value is None:
            env.pop(key, None)
        else:
            env[key] = value
    for key, value in entry["limits"].items():
        if value is not None:
            env[f"SPARKNET_{key}"] = value
    return env


def required_patches(env: dict[str, str]) -> list[str]:
    """NCCL patches an environment needs: none on B200 (stock NCCL)."""
    return [p for key, patches in PATCH_CONTROLS.items() if env.get(key) for p in patches]


def problems(env: dict[str, str], *, world: int) -> list[str]:
    """Settings that contradict each other or the world size."""
    errors: list[str] = []
    for key in ("NCCL_BUFFSIZE", "NCCL_MIN_NCHANNELS", "NCCL_MAX_NCHANNELS", "SPARKNET_TIMEOUT_MS"):
        if key in env and (not str(env[key]).isdigit() or int(env[key]) <= 0):
            errors.append(f"{key} must be a positive integer")
    if str(env.get("NCCL_MAX_NCHANNELS", "")).isdigit() and \
            int(env.get("NCCL_MIN_NCHANNELS", "1") or 1) > int(env["NCCL_MAX_NCHANNELS"]):
        errors.append("NCCL minimum channels exceeds maximum")
    if env.get("NCCL_NET") == "IB" and env.get("NCCL_P2P_DISABLE") == "1" and world > 1:
        errors.append("NCCL is forced onto IB with P2P disabled: inside one NVSwitch box this measures the NIC, "
                      "not NVLink (use it only as the reference's control arm)")
    capacity = env.get("SPARKNET_ALLREDUCE_CAPACITY_BYTES")
    dispatch = env.get("SPARKNET_ALLREDUCE_DISPATCH_MAX_BYTES")
    gather = env.get("SPARKNET_ALLGATHER_MAX_BYTES")
    for label, value in (("all-reduce capacity", capacity), ("all-gather limit", gather),
                         ("all-reduce dispatch", dispatch)):
        if value is not None and (not str(value).isdigit() or int(value) <= 0 or int(value) % 16):
            errors.append(f"{label} must be a positive multiple of 16 bytes")
    if capacity and dispatch and str(capacity).isdigit() and str(dispatch).isdigit() and int(dispatch) > int(capacity):
        errors.append("dispatch limit must not exceed registered capacity")
    if env.get("SPARKNET_NVLS") == "1" and env.get("NCCL_NVLS_ENABLE") == "0":
        errors.append("SPARKNET_NVLS=1 contradicts NCCL_NVLS_ENABLE=0")
    if world not in _WORLDS:
        errors.append(f"world size {world} is not one of {_WORLDS}")
    return errors


__all__ = ["COMMON_ENV", "COMMON_IB_ENV", "PATCH_CONTROLS", "PROFILES", "REFERENCE_IB_ENV", "environment",
           "problems", "profile", "profile_problems", "profiles_for", "required_patches", "size_bytes"]
