"""NVLink adapter for vLLM's CUDA device communicator (one NVSwitch box, TP 2/4/8).

A thin shim with the reference adapter's constructor keywords and methods
(``sparknet/integration/vllm/roce_all_reduce.py:64-275`` of the reference): capability
voting, construction, preparation and size gating live here; the protocol lives in
``sparknet.oneshot``.

- Every rank checks the API version and parses the size limits before the vote; the
  parsed limits travel with the vote and must be identical.  A rank that cannot take
  part aborts initialisation on every rank: selecting this backend is a policy, not a
  request to try other backends on failure.
- Dispatch is rank-invariant: eligibility depends on dtype, shape, contiguity and size,
  never on pointer values.
- Failures are fail-stop: a wait that times out poisons the runtime, later launches
  do nothing, and ``check_health`` (called after each step's host synchronisation)
  raises so the step's output never leaves the worker.
- The group must live on one NVSwitch box (the reference adapter targets the opposite
  case, multi-node groups); a group spanning boxes leaves the adapter disabled.
- ``supports_fused_add_rms_norm()`` is True: ``fused_add_rms_norm`` runs the
  all-reduce, the residual add and RMSNorm in one kernel (bit-identical ranks).
- Setup exchanges go over the CPU (gloo) group; launchers are AOT-compiled and
  ``prepare`` runs at construction, before any graph capture.
"""

from __future__ import annotations

import logging
import os
import re
from collections.abc import Sequence
from contextlib import contextmanager
from dataclasses import dataclass

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)

REQUIRED_API_VERSION = 3
ENV_ALLREDUCE_LIMIT = ("SPARKNET_ALLREDUCE_CAPACITY_BYTES",)
ENV_ALLGATHER_LIMIT = ("SPARKNET_ALLGATHER_MAX_BYTES",)


def parse_byte_size(value: str) -> int:
    """``2MB`` or ``2097152``; KB/MB/GB are binary units, as vLLM parses them."""
    match = re.fullmatch(r"\s*([1-9][0-9]*)\s*(B|KB|MB|GB)?\s*", str(value), re.I)
    if not match:
        raise ValueError(f"invalid byte size {value!r}")
    unit = (match[2] or "B").upper()
    return int(match[1]) * {"B": 1, "KB": 1024, "MB": 1024 ** 2, "GB": 1024 ** 3}[unit]


def _env(names: Sequence[str], default: str | None = None) -> str | None:
    for name in names:
        value = os.environ.get(name)
        if value:
            return value
    return default


@dataclass(frozen=True)
class Readiness:
    """One rank's answer to "can this rank serve the NVLink collectives?": everything
    that stops it (empty when ready) and the size limits it would register."""

    rank: int
    blockers: tuple[str, ...]
    limits: tuple[int, int] | None


def agreement(answers: Sequence[Readiness]) -> str | None:
    """None when every rank is ready with the same limits; otherwise one message that
    names every blocked rank, or every distinct set of limits and the ranks holding it.
    Pure function of the gathered answers, so every rank reaches the same verdict."""
    blocked = [f"rank {a.rank} cannot serve: {'; '.join(a.blockers)}" for a in answers if a.blockers]
    if blocked:
        return " | ".join(blocked)
    holders: dict[tuple[int, int] | None, list[int]] = {}
    for a in answers:
        holders.setdefault(a.limits, []).append(a.rank)
    if len(holders) > 1:
        spread = ", ".join(f"ranks {ranks}: all-reduce {lim[0]} B / all-gather {lim[1]} B" if lim else
                           f"ranks {ranks}: none" for lim, ranks in holders.items())
        return f"size limits disagree across ranks ({spread})"
    return None


class SparknetOneShotAllReduce:
    """Route eligible tensor-parallel collectives to ``sparknet.oneshot`` over NVLink."""

    backend_name = "SPARKNET_NVLINK"

    def __init__(self, group, device_group, device: torch.device, *, global_ranks: Sequence[int] | None = None,
                 nccl_available: bool = True, in_the_same_node: Sequence[bool] | None = None,
                 runtime_factory=None) -> None:
        self.group, self.device_group, self.device = group, device_group, device
        self.rank = dist.get_rank(group=group)
        self.world_size = dist.get_world_size(group=group)
        self.global_ranks = tuple(range(self.world_size)) if global_ranks is None else tuple(map(int, global_ranks))
        self._runtime = None
        self._announced: set[str] = set()
        self.disabled = True
        if len(self.global_ranks) != self.world_size:
            raise ValueError(f"{len(self.global_ranks)} global ranks for a group of {self.world_size}")
        if device_group is None:
            raise RuntimeError("the NVLink adapter needs the CUDA (NCCL) process group beside the CPU group")
        if in_the_same_node is not None and not all(in_the_same_node):
            # every rank sees the same list, so every rank leaves the adapter off here
            logger.info("NVLink collectives off: the tensor-parallel group spans several boxes")
            return
        mine = self._assess()
        if not nccl_available:
            mine = Readiness(mine.rank, mine.blockers + ("NCCL must stay available for ineligible inputs",),
                             mine.limits)
        answers: list = [None] * self.world_size
        dist.all_gather_object(answers, mine, group=self.group)
        verdict = agreement(answers)
        if verdict is not None:
            raise RuntimeError(f"NVLink collective policy unavailable: {verdict}")
        capacity, gather_shard = mine.limits
        factory = runtime_factory
        if factory is None:
            from sparknet import oneshot

            factory = oneshot.AllReduce.from_exchange_group
        try:
            runtime = factory(exchange_group=group, device=device, max_size=capacity, max_gather_bytes=gather_shard)
            runtime.prepare((torch.float16, torch.bfloat16, torch.float32), padded_gather=True)
        except Exception as exc:  # noqa: BLE001 - the runtime's own set-up is collective
            raise RuntimeError("NVLink collective initialization failed") from exc
        self._runtime, self.disabled = runtime, False
        if self.rank == 0:
            logger.info("NVLink collectives on (world %d): all-reduce up to %d B of a %d B capacity, all-gather "
                        "shards up to %d B, fused add + RMSNorm; NCCL carries the rest; a failure is fatal",
                        self.world_size, self.all_reduce_max_bytes, self.all_reduce_capacity_bytes,
                        self.all_gather_max_bytes)

    def _assess(self) -> Readiness:
        """Everything that stops this rank, checked in full (not just the first)."""
        blockers: list[str] = []
        limits = None
        try:
            capacity = parse_byte_size(_env(ENV_ALLREDUCE_LIMIT, "8MB"))
            gather_shard = parse_byte_size(_env(ENV_ALLGATHER_LIMIT, "16MB"))
            limits = (capacity, gather_shard)
        except ValueError as exc:
            blockers.append(f"size limit: {exc}")
        try:
            from sparknet import oneshot
        except ImportError as exc:
            blockers.append(f"sparknet.oneshot does not import ({exc})")
            return Readiness(self.rank, tuple(blockers), limits)
        api = getattr(oneshot, "API_VERSION", None)
        if api != REQUIRED_API_VERSION:
            blockers.append(f"sparknet.oneshot speaks API {api}, this adapter speaks {REQUIRED_API_VERSION}")
        elif not oneshot.is_supported(self.device):
            blockers.append(f"{self.device} is not a B200 (sm_100) with the sparknet extension built")
        return Readiness(self.rank, tuple(blockers), limits)

    def _announce(self, kind: str, message: str, *args) -> None:
        if kind in self._announced:
            return
        self._announced.add(kind)
        (logger.info if self.rank == 0 else logger.debug)(message, *args)

    # -- policy surface ------------------------------------------------------------------
    @property
    def all_reduce_max_bytes(self) -> int:
        return 0 if self.disabled else int(self._runtime.dispatch_max_bytes)

    @property
    def all_reduce_capacity_bytes(self) -> int:
        return 0 if self.disabled else int(self._runtime.max_size)

    @property
    def all_gather_max_bytes(self) -> int:
        return 0 if self.disabled else int(self._runtime.max_gather_bytes)

    def check_health(self) -> None:
        if not self.disabled and self._runtime is not None:
            self._runtime.check_health()

    def failure(self) -> str | None:
        return None if self.disabled or self._runtime is None else self._runtime.failure()

    def should_custom_ar(self, inp: torch.Tensor) -> bool:
        return not self.disabled and self._runtime.should_allreduce(inp)

    def custom_all_reduce(self, inp: torch.Tensor) -> torch.Tensor | None:
        if not self.should_custom_ar(inp):
            return None
        self._announce("ar", "NVLink all-reduce is live: first routed all-reduce is %d bytes (%s)",
                       inp.numel() * inp.element_size(), str(inp.dtype).replace("torch.", ""))
        return self._runtime.all_reduce(inp)

    def supports_fused_add_rms_norm(self) -> bool:
        return not self.disabled

    def should_fused_add_rms_norm(self, inp: torch.Tensor, residual: torch.Tensor) -> bool:
        if self.disabled or inp.dim() != 2 or residual.shape != inp.shape or inp.dtype != residual.dtype:
            return False
        return self._runtime.should_allreduce(inp) and residual.is_contiguous() and inp.shape[1] % 64 == 0

    def fused_add_rms_norm(self, inp: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float) -> tuple[torch.Tensor, torch.Tensor]:
        """``residual = all_reduce(inp) + residual; out = rms_norm(residual) * weight``: returns
        ``(out, residual)`` with the residual updated in place, as vLLM's fused op does."""
        self._announce("fused", "NVLink fused all-reduce + RMSNorm is live: first routed tensor %s",
                       tuple(inp.shape))
        out, _ = self._runtime.all_reduce_residual_rmsnorm(inp, residual, weight, eps, residual_out=residual)
        return out, residual

    def should_all_gather(self, inp: torch.Tensor, dim: int) -> bool:
        return not self.disabled and self._runtime.should_all_gather(inp, dim)

    def all_gather(self, inp: torch.Tensor, dim: int) -> torch.Tensor:
        self._announce("ag", "NVLink all-gather is live: first routed shard is %s along dim %d", tuple(inp.shape), dim)
        return self._runtime.all_gather(inp, dim=dim)

    def should_reduce_scatter(self, inp: torch.Tensor, dim: int = 0) -> bool:
        return (not self.disabled and inp.numel() * inp.element_size() <= self._runtime.max_size
                and self._runtime.should_reduce_scatter(inp, dim=dim))

    def reduce_scatter(self, inp: torch.Tensor, dim: int = 0) -> torch.Tensor:
        self._announce("rs", "NVLink reduce-scatter is live: first routed input is %s", tuple(inp.shape))
        return self._runtime.reduce_scatter(inp, dim=dim)

    def should_exchange(self, chunks: torch.Tensor, parts: torch.Tensor | None = None) -> bool:
        return (not self.disabled and chunks.numel() * chunks.element_size() <= self.world_size * self.all_gather_max_bytes
                and self._runtime.should_exchange(chunks, parts))

    def exchange_into(self, chunks: torch.Tensor, parts: torch.Tensor) -> torch.Tensor:
        self._announce("ex", "NVLink exchange is live: first routed tensor is %s", tuple(chunks.shape))
        return self._runtime.exchange(chunks, out=parts)

    def should_all_to_all_rows(self, inp: torch.Tensor, rows: int) -> bool:
        return not self.disabled and self._runtime.should_all_to_all_rows(inp, rows)

    def all_to_all_rows(self, inp: torch.Tensor, rows: int) -> torch.Tensor:
        self._announce("a2a", "NVLink all-to-all rows is live: first routed tensor is %s", tuple(inp.shape))
        return self._runtime.all_to_all_rows(inp, rows)

    @contextmanager
    def capture(self, stream: torch.cuda.Stream | None = None):
        if self.disabled:
            yield
            return
        with self._runtime.capture(stream=stream):
            yield

    def close(self) -> None:
        if self._runtime is not None:
            self._runtime.close()
            self._runtime = None
        self.disabled = True


__all__ = ["REQUIRED_API_VERSION", "Readiness", "SparknetOneShotAllReduce", "agreement", "parse_byte_size"]
