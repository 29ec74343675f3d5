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


class SparknetOneShotAllReduce:
    """Route eligible tensor-parallel collectives to ``sparknet.oneshot`` over NVLink."""

    backend_name = "SPARKNET_NVLINK"

    def __init__(self, group, device_group, device: torch.device, *, global_ranks: Sequence[int] | None = None,
                 nccl_available: bool = True, in_the_same_node: Sequence[bool] | None = None,
                 runtime_factory=None) -> None:
        self.disabled = True
        self.group = group
        self.device_group = device_group
        self.device = device
        self.rank = dist.get_rank(group=group)
        self.world_size = dist.get_world_size(group=group)
        self._runtime = None
        self._announced: set[str] = set()
        self.global_ranks = tuple(int(r) for r in (global_ranks if global_ranks is not None
                                                   else range(self.world_size)))
        if len(self.global_ranks) != self.world_size:
            raise ValueError("global ranks must match the process group")
        if device_group is None:
            raise RuntimeError("the NVLink adapter requires a CUDA process group")
        if in_the_same_node is not None and not all(in_the_same_node):
            logger.info("NVLink collectives skipped: the group spans more than one box")
            return
        reason, limits = self._local_capability()
        if not nccl_available:
            reason = "the policy requires an available NCCL communicator"
        verdict = self._exchange_vote(reason, limits)
        if verdict is not None:
            raise RuntimeError(f"NVLink collective policy unavailable: {verdict}")
        max_size, max_gather = limits
        if runtime_factory is None:
            from sparknet import oneshot

            runtime_factory = oneshot.AllReduce.from_exchange_group
        try:
            self._runtime = runtime_factory(exchange_group=group, device=device, max_size=max_size,
                                            max_gather_bytes=max_gather)
            self._runtime.prepare((torch.float16, torch.bfloat16, torch.float32), padded_gather=True)
        except Exception as exc:  # noqa: BLE001 - the runtime already coordinated ranks
            raise RuntimeError("NVLink collective initialization failed") from exc
        self.disabled = False
        if self.rank == 0:
            logger.info("Using NVLink collectives: world=%d, all-reduce dispatch <=%d bytes, capacity=%d bytes, "
                        "all-gather shard <=%d bytes, fused add+RMSNorm on. NCCL handles ineligible inputs; "
                        "failures are fatal.", self.world_size, self.all_reduce_max_bytes,
                        self.all_reduce_capacity_bytes, self.all_gather_max_bytes)

    def _local_capability(self):
        try:
            from sparknet import oneshot
        except ImportError as exc:
            return f"sparknet.oneshot is not importable: {exc}", None
        api = getattr(oneshot, "API_VERSION", None)
        if api != REQUIRED_API_VERSION:
            return f"sparknet.oneshot API version {api}, adapter needs {REQUIRED_API_VERSION}", None
        if not oneshot.is_supported(self.device):
            return "needs a B200 (compute capability 10.0) with the sparknet extension built", None
        try:
            limits = (parse_byte_size(_env(ENV_ALLREDUCE_LIMIT, "8MB")),
                      parse_byte_size(_env(ENV_ALLGATHER_LIMIT, "16MB")))
        except Exception as exc:  # noqa: BLE001 - reported through the vote
            return f"invalid size limit: {exc}", None
        return None, limits

    def _exchange_vote(self, reason, limits):
        votes = [(None, None)] * self.world_size
        dist.all_gather_object(votes, (reason, limits), group=self.group)
        failures = [f"rank {i}: {r}" for i, (r, _) in enumerate(votes) if r]
        if failures:
            return "; ".join(failures)
        reference = votes[0][1]
        differing = [f"rank {i}: {lim}" for i, (_, lim) in enumerate(votes) if lim != reference]
        if differing:
            return f"size limits differ across ranks (rank 0: {reference}; " + "; ".join(differing) + ")"
        return None

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


__all__ = ["REQUIRED_API_VERSION", "SparknetOneShotAllReduce", "parse_byte_size"]
