"""One collective policy, fixed before any graph capture.

Which transport carries each collective is decided from the operation, dtype,
contiguity, byte size and world size only: values every tensor-parallel rank
shares, never pointer values or timing, so every rank routes the same call the same
way.  A transport failure is a coordinated failure, never a local switch to another
backend (fail-stop).

The reference (``sparknet/policy/policy.py:34-114``) has two backends: its one-shot
RDMA collectives or NCCL.  On an NVSwitch box there are four:

- ``oneshot``: every rank pushes its whole input into every peer (latency-optimal,
  W-1 times the message crosses each rank's NVLink);
- ``twoshot``: reduce-scatter then all-gather over pushes (2(W-1)/W of the message
  per rank; bandwidth-optimal for mid-size messages);
- ``nvls``: NVLink SHARP in-switch reduction with ``multimem`` (opt-in: the switch's
  summation order is not the rank order, so results are rank-identical but not
  equal to the sequential fp32 reference);
- ``nccl``: everything above the registered capacity, and every ineligible tensor.

Three limits stay distinct, as in the reference:

- the all-reduce **dispatch** ceiling: the largest message sent to the custom kernels;
- the all-reduce **capacity**: the registered slot size (may exceed dispatch; vLLM's
  sequence-parallel threshold reads it);
- the all-gather limit on the **input shard**.

The one-shot/two-shot crossover is a per-world-size table measured on B200
(``sparknet probe collectives --benchmark`` writes one; ``crossover_from_timings``
turns its timings into a table).
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Mapping

PACK_BYTES = 16
SUPPORTED_DTYPES = ("float16", "bfloat16", "float32")
_GATHER_REJECTED_DTYPES = ("bool", "complex64", "complex128")
BACKENDS = ("oneshot", "twoshot", "nvls", "nccl")
GATHER_ALGORITHMS = ("ll", "push", "nvls")

ENV_CAPACITY = "SPARKNET_ALLREDUCE_CAPACITY_BYTES"
ENV_DISPATCH = "SPARKNET_ALLREDUCE_DISPATCH_MAX_BYTES"
ENV_GATHER = "SPARKNET_ALLGATHER_MAX_BYTES"
ENV_CROSSOVER = "SPARKNET_ONESHOT_MAX_BYTES"
ENV_ALGO = "SPARKNET_ALGO"
ENV_NVLS = "SPARKNET_NVLS"

# Largest all-reduce (bytes per rank) that one-shot carries, by world size, and the
# all-reduce dispatch ceiling, by world size.  Both come from the committed sweep
# (``measured_b200.json`` beside this module, made by ``sparknet probe collectives
# --benchmark --sweep`` on B200 boxes and ``sparknet policy derive``); they are read
# once at import, so every rank of a job holds the same values.  Without the file the
# fallbacks below apply (an earlier W=8 measurement: one-shot 11.9 us vs two-shot
# 14.5 us at 480 KiB, 17.5 vs 15.1 us at 1 MiB).
FALLBACK_ONESHOT_MAX = {2: 4 << 20, 4: 512 << 10, 8: 512 << 10}
FALLBACK_DISPATCH_MAX = 2 << 20
# Largest all-gather shard that travels in LL8 form (payload + flag per 8 bytes);
# larger shards use bulk pushes with per-block flags (or NVLS broadcast when enabled).
# LL doubles the bytes but needs no fence or flag round trip.  The default is derived
# from the committed table (``ll_max`` of the worlds whose sweep timed the all-gather
# protocols separately; on 2 B200s LL beat the push, NVLS and NCCL up to its 4 MiB slot,
# 20.7 against 23.1 / 41.1 / 39.5 us at 4 MiB); this fallback applies without it.  On 8
# B200s LL beat NCCL up to 4 MiB (105.4 vs 113.0 us) and lost at 8 MiB (211.0 vs 195.8).
FALLBACK_LL_MAX = 4 << 20
# Messages at or above this use NVLS when it is enabled and available (the measured
# threshold of the smallest world size that has one, else this fallback).
FALLBACK_NVLS_MIN = 256 << 10


@dataclass(frozen=True)
class CollectivePolicy:
    all_reduce_dispatch_bytes: int
    all_reduce_capacity_bytes: int
    all_gather_shard_bytes: int
    oneshot_max_bytes: Mapping[int, int] = field(default_factory=lambda: dict(DEFAULT_ONESHOT_MAX))  # noqa: F821
    ll_max_bytes: int = field(default_factory=lambda: DEFAULT_LL_MAX)
    allow_nvls: bool = False
    nvls_min_bytes: int = field(default_factory=lambda: DEFAULT_NVLS_MIN)  # noqa: F821
    force: str | None = None

    def problems(self) -> list[str]:
        errors = []
        for label, value in (("all_reduce_dispatch_bytes", self.all_reduce_dispatch_bytes),
                             ("all_reduce_capacity_bytes", self.all_reduce_capacity_bytes),
                             ("all_gather_shard_bytes", self.all_gather_shard_bytes)):
            if value < PACK_BYTES or value % PACK_BYTES:
                errors.append(f"{label} must be a multiple of {PACK_BYTES} bytes, at least {PACK_BYTES}")
        if self.all_reduce_dispatch_bytes > self.all_reduce_capacity_bytes:
            errors.append("all-reduce dispatch must not exceed registered capacity")
        if self.force is not None and self.force not in BACKENDS:
            errors.append(f"{ENV_ALGO} must be one of {BACKENDS}, got {self.force!r}")
        if self.force == "nvls" and not self.allow_nvls:
            errors.append(f"{ENV_ALGO}=nvls needs {ENV_NVLS}=1 (NVLS sums are not in rank order)")
        for world, limit in self.oneshot_max_bytes.items():
            if int(world) < 1 or int(limit) < 0:
                errors.append(f"one-shot crossover for world {world} must be a non-negative byte count")
        return errors

    # -- all-reduce --------------------------------------------------------------
    def all_reduce_eligible(self, nbytes: int, dtype: str, *, contiguous: bool = True) -> bool:
        return (contiguous and dtype in SUPPORTED_DTYPES and 0 < nbytes <= self.all_reduce_dispatch_bytes
                and nbytes % PACK_BYTES == 0)

    def all_reduce_backend(self, nbytes: int, dtype: str, *, contiguous: bool = True, world: int = 8) -> str:
        """``oneshot``, ``twoshot`` or ``nvls`` for an eligible input, else ``nccl``."""
        if not self.all_reduce_eligible(nbytes, dtype, contiguous=contiguous):
            return "nccl"
        if self.force is not None:
            return self.force
        if world <= 1:
            return "oneshot"
        if self.allow_nvls and nbytes >= self.nvls_min_bytes:
            return "nvls"
        return "oneshot" if nbytes <= self.oneshot_limit(world) else "twoshot"

    def oneshot_limit(self, world: int) -> int:
        if world in self.oneshot_max_bytes:
            return int(self.oneshot_max_bytes[world])
        # between measured sizes: the nearest smaller world's limit
        smaller = [w for w in self.oneshot_max_bytes if w <= world]
        return int(self.oneshot_max_bytes[max(smaller)]) if smaller else 0

    # -- all-gather --------------------------------------------------------------
    def all_gather_backend(self, shard_bytes: int, dtype: str, *, dim: int, ndim: int,
                           contiguous: bool = True) -> str:
        """``oneshot`` (a custom kernel) for a contiguous shard concatenated along dim 0
        or the last dim within the limit, else ``nccl``."""
        if dim < 0:
            dim += ndim
        if (contiguous and ndim > 0 and dtype not in _GATHER_REJECTED_DTYPES and dim in (0, ndim - 1)
                and 0 < shard_bytes <= self.all_gather_shard_bytes):
            return "oneshot"
        return "nccl"

    def all_gather_algorithm(self, shard_bytes: int, *, row_bytes: int, nvls_available: bool) -> str:
        """Which custom all-gather kernel: ``ll``, ``push`` or ``nvls`` (all rank-invariant)."""
        if shard_bytes <= self.ll_max_bytes and shard_bytes % 8 == 0 and row_bytes % 8 == 0:
            return "ll"
        if self.allow_nvls and nvls_available and shard_bytes >= self.nvls_min_bytes:
            return "nvls"
        return "push"

    @staticmethod
    def reduce_scatter_backend(nbytes: int = 0, capacity: int | None = None) -> str:
        """Reduce-scatter uses the custom kernel within capacity, NCCL above it."""
        if capacity is not None and 0 < nbytes <= capacity:
            return "oneshot"
        return "nccl"

    # -- environment round trip ----------------------------------------------------
    def environment(self) -> dict[str, str]:
        env = {
            ENV_CAPACITY: str(self.all_reduce_capacity_bytes),
            ENV_DISPATCH: str(self.all_reduce_dispatch_bytes),
            ENV_GATHER: str(self.all_gather_shard_bytes),
            ENV_CROSSOVER: json.dumps({str(k): int(v) for k, v in sorted(self.oneshot_max_bytes.items())
                                       if v < (1 << 62)}),
        }
        if self.allow_nvls:
            env[ENV_NVLS] = "1"
        if self.force:
            env[ENV_ALGO] = self.force
        return env

    @classmethod
    def from_environment(cls, env: Mapping[str, str]) -> "CollectivePolicy":
        """Read the limits, in bytes, as a recipe sets them."""
        capacity = env.get(ENV_CAPACITY)
        gather = env.get(ENV_GATHER)
        if not capacity or not gather:
            raise ValueError("the environment names no all-reduce capacity or all-gather limit")
        dispatch = env.get(ENV_DISPATCH) or capacity
        crossovers = dict(DEFAULT_ONESHOT_MAX)
        if env.get(ENV_CROSSOVER):
            crossovers.update({int(k): int(v) for k, v in json.loads(env[ENV_CROSSOVER]).items()})
        policy = cls(int(dispatch), int(capacity), int(gather), oneshot_max_bytes=crossovers,
                     allow_nvls=env.get(ENV_NVLS, "0") not in ("", "0", "false", "False"),
                     force=env.get(ENV_ALGO) or None)
        errors = policy.problems()
        if errors:
            raise ValueError("; ".join(errors))
        return policy


# -- limits derived from a committed measurement ------------------------------------
MEASURED_TABLE = Path(__file__).with_name("measured_b200.json")


@dataclass(frozen=True)
class MeasuredLimits:
    """Per-world-size limits derived from latency sweeps.

    - ``oneshot_max``: the largest size up to which one-shot is never slower than
      two-shot (the one-shot / two-shot crossover);
    - ``dispatch_max``: the largest size up to which the faster NVLink arm is never
      slower than NCCL (the all-reduce dispatch ceiling);
    - ``nvls_min``: the smallest size from which NVLS beats both push arms at every
      measured size (None when NVLS was not measured or never wins);
    - ``ll_max``: the largest all-gather shard up to which the LL8 protocol is never
      slower than any other all-gather arm (only worlds whose sweep timed the
      protocols separately).
    """

    oneshot_max: Mapping[int, int]
    dispatch_max: Mapping[int, int]
    nvls_min: Mapping[int, int | None]
    ll_max: Mapping[int, int] = field(default_factory=dict)


SWEPT_OPERATIONS = ("all_reduce", "all_gather")


def sweep_rows(receipt: Mapping, world: int) -> list[dict]:
    """All-reduce and all-gather rows of a probe receipt (``sparknet probe collectives
    --benchmark --sweep``) as ``{world, nbytes, arm, p50_us}`` (plus ``operation`` for
    the all-gather); the arm is the backend the case ran on (a forced arm outside its
    range ran elsewhere and is dropped).  All-gather rows count only when the sweep
    timed its protocols (``ll``, ``push``, ``nvls``) as separate arms."""
    item = {"bfloat16": 2, "float16": 2, "float32": 4}
    out = []
    for row in receipt.get("timings", ()):
        operation = row.get("operation")
        if operation not in SWEPT_OPERATIONS or row.get("arm") == "policy":
            continue
        if row.get("backend", row["arm"]) != row["arm"]:
            continue
        if operation == "all_gather" and row["arm"] not in ("ll", "push", "nvls", "nccl"):
            continue
        dtype = str(row["dtype"]).rsplit(".", 1)[-1]
        entry = {"world": int(world), "nbytes": int(row["elements_per_rank"]) * item[dtype], "arm": row["arm"],
                 "p50_us": float(row["median_us"])}
        if operation != "all_reduce":
            entry["operation"] = operation
        out.append(entry)
    return out


def _by_world_size(rows, operation: str = "all_reduce") -> dict[int, dict[int, dict[str, float]]]:
    table: dict[int, dict[int, dict[str, float]]] = {}
    for row in rows:
        if row.get("operation", "all_reduce") != operation:
            continue
        table.setdefault(int(row["world"]), {}).setdefault(int(row["nbytes"]), {})[row["arm"]] = float(row["p50_us"])
    return table


def derive_limits(rows) -> MeasuredLimits:
    """``MeasuredLimits`` from sweep rows (``{world, nbytes, arm, p50_us}``).

    Each limit is taken from the smallest size upward and stops at the first size that
    breaks it, so a limit never skips over a size where its arm lost."""
    oneshot, dispatch, nvls = {}, {}, {}
    for world, sizes in _by_world_size(rows).items():
        one_lim, disp_lim, nvls_from = 0, 0, None
        one_open = disp_open = True
        for nbytes in sorted(sizes):
            arms = sizes[nbytes]
            push = [arms[a] for a in ("oneshot", "twoshot") if a in arms]
            if one_open and "oneshot" in arms:
                if "twoshot" not in arms or arms["oneshot"] <= arms["twoshot"]:
                    one_lim = nbytes
                else:
                    one_open = False
            if disp_open and push and "nccl" in arms:
                if min(push) <= arms["nccl"]:
                    disp_lim = nbytes
                else:
                    disp_open = False
            if "nvls" in arms and push:
                if arms["nvls"] < min(push):
                    nvls_from = nvls_from if nvls_from is not None else nbytes
                else:
                    nvls_from = None
        oneshot[world], dispatch[world], nvls[world] = one_lim, disp_lim, nvls_from
    ll = {}
    for world, sizes in _by_world_size(rows, "all_gather").items():
        # only sizes at which the protocols themselves were timed (a receipt of another
        # sweep may add NCCL-only rows at other sizes)
        timed = [n for n in sorted(sizes) if any(a in sizes[n] for a in ("ll", "push", "nvls"))]
        if not timed:
            continue
        ll_lim = 0
        for nbytes in timed:
            arms = sizes[nbytes]
            others = [v for a, v in arms.items() if a != "ll"]
            if "ll" not in arms or (others and arms["ll"] > min(others)):
                break  # beyond the LL slot, or LL lost: the limit stops here
            ll_lim = nbytes
        ll[world] = ll_lim
    return MeasuredLimits(oneshot, dispatch, nvls, ll)


def load_measured(path: str | Path | None = None) -> MeasuredLimits | None:
    """The limits derived from the committed sweep (``measured_b200.json`` beside this
    module), or None if it is absent."""
    target = Path(path) if path is not None else MEASURED_TABLE
    if not target.exists():
        return None
    return derive_limits(json.loads(target.read_text())["rows"])


def crossover_from_timings(rows: list[dict]) -> dict[int, int]:
    """The largest size at which one-shot beat two-shot, per world size.

    ``rows`` are probe timing rows with ``world_size``, ``nbytes``, ``algorithm`` and
    ``p50_us`` keys.  Sizes are compared pairwise; the crossover is the largest size
    below the first size where two-shot wins.
    """
    table: dict[int, int] = {}
    by_world: dict[int, dict[int, dict[str, float]]] = {}
    for row in rows:
        by_world.setdefault(int(row["world_size"]), {}).setdefault(int(row["nbytes"]), {})[row["algorithm"]] = \
            float(row["p50_us"])
    for world, sizes in by_world.items():
        limit = 0
        for nbytes in sorted(sizes):
            arms = sizes[nbytes]
            if "oneshot" not in arms or "twoshot" not in arms:
                continue
            if arms["oneshot"] <= arms["twoshot"]:
                limit = nbytes
            else:
                break
        table[world] = limit
    return table


_MEASURED = load_measured()
DEFAULT_ONESHOT_MAX = {1: 1 << 62, **FALLBACK_ONESHOT_MAX,
                       **({w: v for w, v in _MEASURED.oneshot_max.items()} if _MEASURED else {})}
_DISPATCH_BY_WORLD = dict(_MEASURED.dispatch_max) if _MEASURED else {}
_nvls = sorted((w, v) for w, v in (_MEASURED.nvls_min.items() if _MEASURED else ()) if v)
DEFAULT_NVLS_MIN = _nvls[0][1] if _nvls else FALLBACK_NVLS_MIN
_ll = [v for v in (_MEASURED.ll_max.values() if _MEASURED else ()) if v]
DEFAULT_LL_MAX = min(_ll) if _ll else FALLBACK_LL_MAX  # the smallest measured limit holds for every world


def default_dispatch_bytes(world: int) -> int:
    """The all-reduce dispatch ceiling for ``world`` ranks: the measured one for that
    world size, else ``FALLBACK_DISPATCH_MAX`` (a ceiling is not extrapolated across
    world sizes); never below 16 bytes."""
    if world in _DISPATCH_BY_WORLD:
        return max(PACK_BYTES, int(_DISPATCH_BY_WORLD[world]))
    return FALLBACK_DISPATCH_MAX


# Profiles for one B200 box: the product (NVLink kernels below 2 MiB dispatch,
# 8 MiB registered capacity, 16 MiB gather shards).
NVLINK_POLICY = CollectivePolicy(2 * 1024 * 1024, 8 * 1024 * 1024, 16 * 1024 * 1024)


def policy_for_profile(name: str) -> CollectivePolicy | None:
    """The policy a named profile sets; None for an NCCL-only profile."""
    from sparknet.nccl.profiles import profile

    limits = profile(name)["limits"]
    if limits["ALLREDUCE_CAPACITY_BYTES"] is None:
        return None
    capacity = int(limits["ALLREDUCE_CAPACITY_BYTES"])
    dispatch = int(limits["ALLREDUCE_DISPATCH_MAX_BYTES"] or capacity)
    return CollectivePolicy(dispatch, capacity, int(limits["ALLGATHER_MAX_BYTES"]))


__all__ = [
    "BACKENDS", "DEFAULT_NVLS_MIN", "DEFAULT_ONESHOT_MAX", "GATHER_ALGORITHMS", "MEASURED_TABLE",
    "default_dispatch_bytes", "PACK_BYTES", "SUPPORTED_DTYPES", "CollectivePolicy",
    "MeasuredLimits", "NVLINK_POLICY", "crossover_from_timings", "derive_limits", "load_measured",
    "policy_for_profile", "sweep_rows",
]
