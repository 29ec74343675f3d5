"""NVLink collective runtime for tensor-parallel inference on one B200 box.

Public surface kept from the reference (``sparknet/oneshot/runtime.py:428-1819``):
``AllReduce.from_exchange_group``, ``prepare``, ``should_allreduce`` /
``all_reduce``, ``should_all_gather`` / ``all_gather``, ``should_reduce_scatter`` /
``reduce_scatter``, ``should_exchange`` / ``exchange``, ``should_all_to_all_rows`` /
``all_to_all_rows``, ``capture``, ``check_health``, ``failure``, ``poisoned``,
``set_timeout_ms``, ``stats``, ``close``.  Added: ``all_reduce_residual_rmsnorm``
(fused decode epilogue), ``reset`` and ``barrier``.

Mechanism.  Each rank owns one symmetric region in its own HBM that every peer has
mapped (``symm.build_regions``).  A collective is one kernel launch on the caller's
stream: the kernel reads this rank's device-resident epoch, pushes data into the
peers' regions with NVLink stores, waits on data-borne arrival markers (Lamport
sentinels or LL flags) or per-block flags in its own memory, reduces in fixed rank
order with fp32 accumulation and bumps the epoch.  Nothing is baked into a launch
that changes between calls, so graphs replay.

Contract (as in the reference):

* one collective in flight per runtime; launches on different streams are ordered
  with an event, captures must use one stream;
* the choice of kernel depends only on dtype, shape, contiguity, size and world
  (rank-invariant), never on pointer values;
* a failed wait records a report in pinned host memory and poisons the runtime;
  later collectives raise before launching (fail-stop, no fallback).  Unlike the
  reference the GPU is not stopped (no ``trap``): the kernel returns, the context
  stays usable and ``reset()`` re-arms the runtime collectively.
"""

from __future__ import annotations

import contextlib
import ctypes
import logging
import os
import threading
from contextlib import contextmanager
from typing import Any, Optional, Sequence

import torch
import torch.distributed as dist

from .. import _native
from ..policy import CollectivePolicy
from ..policy.policy import (DEFAULT_ONESHOT_MAX, ENV_ALGO, ENV_CROSSOVER, ENV_NVLS, PACK_BYTES,
                             default_dispatch_bytes)
from . import symm, trace
from ._freeze import raise_if_kernel_resolution_frozen

logger = logging.getLogger(__name__)

API_VERSION = 3
SUPPORTED_DTYPES = (torch.float16, torch.bfloat16, torch.float32)
SUPPORTED_WORLD_SIZES = (1, 2, 3, 4, 5, 6, 7, 8)
TOPOLOGIES = ("nvswitch",)
DEFAULT_MAX_SIZE = 8 * 1024 * 1024
DEFAULT_MAX_GATHER_BYTES = 16 * 1024 * 1024
DEFAULT_THREADS = 512
DEFAULT_BLOCKS = 0          # 0: one block per SM at most
DEFAULT_TIMEOUT_MS = 10_000
MAX_TIMEOUT_MS = (2**32 - 1) // 1000
LL_CAP = 4 * 1024 * 1024   # LL8 slot: all-gather shards up to this travel as payload + flags

ALGO_CODES = {"oneshot": 0, "twoshot": 1, "nvls": 2, "local": 3}
GATHER_CODES = {"ll": 0, "push": 1, "nvls": 2}
FAIL_KINDS = {1: "timed out", 2: "was poisoned", 3: "exceeded its poll limit",
              4: "accessed a slot out of bounds (bounds-checked build)",
              5: "found a launch shape it cannot serve"}
OP_NAMES = {1: "all-reduce", 2: "all-gather", 3: "reduce-scatter", 4: "exchange", 5: "barrier",
            6: "fused all-reduce+RMSNorm"}

ENV_TIMEOUT_MS = "SPARKNET_TIMEOUT_MS"
ENV_PDL = "SPARKNET_PDL"
ENV_DISPATCH = "SPARKNET_ALLREDUCE_DISPATCH_MAX_BYTES"
# Settings of the reference's RoCE transport have no meaning on NVLink; refused with
# the reason instead of silently ignored.
REMOVED_SETTINGS = {
    "SPARKNET_ROCE_TOPOLOGY": "there is no cabling mode on an NVSwitch box",
    "SPARKNET_ROCE_HCA": "the transport is NVLink, not an RDMA device",
    "SPARKNET_ROCE_PEER_HCAS": "the transport is NVLink, not an RDMA device",
    "SPARKNET_ROCE_SUBNETS": "peers are identified by GPU, not by subnet",
    "SPARKNET_ROCE_GID_INDEX": "peers are identified by GPU, not by GID",
    "SPARKNET_ROCE_SPIN_LIMIT": "waits are timed: set SPARKNET_TIMEOUT_MS",
    "SPARKNET_ROCE_TIMEOUT_MS": "renamed: set SPARKNET_TIMEOUT_MS",
    "SPARKNET_ROCE_ALLREDUCE_CAPACITY_BYTES": "renamed: set SPARKNET_ALLREDUCE_CAPACITY_BYTES",
    "SPARKNET_ROCE_ALLREDUCE_DISPATCH_MAX_BYTES": "renamed: set SPARKNET_ALLREDUCE_DISPATCH_MAX_BYTES",
    "SPARKNET_ROCE_ALLGATHER_MAX_BYTES": "renamed: set SPARKNET_ALLGATHER_MAX_BYTES",
    "SPARKNET_ROCE_PROXY_CPU": "there is no host proxy",
    "SPARKNET_ROCE_MESH_ROTATE": "there is no mesh routing on NVSwitch",
    "SPARKNET_ROCE_TRACE": "renamed: set SPARKNET_TRACE",
}


def removed_setting_problems(environ) -> list[str]:
    return [f"{name} is not read by this build: {why}" for name, why in REMOVED_SETTINGS.items()
            if environ.get(name)]


def checked_timeout_ms(value: int) -> int:
    value = int(value)
    if not 1 <= value <= MAX_TIMEOUT_MS:
        raise ValueError(f"the collective wait timeout must be 1 to {MAX_TIMEOUT_MS} ms, got {value}")
    return value


def is_supported(device: torch.device | int | str | None = None) -> bool:
    """True on a CUDA device of compute capability 10.0 (B200) with the extension built."""
    if not torch.cuda.is_available():
        return False
    index = torch.cuda.current_device() if device is None else torch.device(device).index
    major, minor = torch.cuda.get_device_capability(index if index is not None else 0)
    return (major, minor) == (10, 0) and _native.available()


def discover_hcas() -> tuple[str, ...]:
    """The RDMA devices the collectives would use: always none on an NVSwitch box.

    The reference picks up to two active RoCE v2 HCAs here (reference
    ``sparknet/oneshot/runtime.py:168-189``) because its one-shot path writes over
    RDMA.  Here every byte of a collective crosses NVLink from inside the kernels, so
    no RDMA device takes part; the name stays importable for code written against the
    reference.  The NVLink devices are :func:`discover_nvlink_gpus`.
    """
    return ()


def discover_nvlink_gpus() -> tuple[int, ...]:
    """CUDA device indices this process can use for the NVLink collectives: B200s
    (compute capability 10.0) that reach every other listed device peer to peer."""
    if not torch.cuda.is_available():
        return ()
    gpus = [i for i in range(torch.cuda.device_count()) if torch.cuda.get_device_capability(i) == (10, 0)]
    return tuple(i for i in gpus if all(i == j or torch.cuda.can_device_access_peer(i, j) for j in gpus))


def normalize_device(device: torch.device | int | str) -> torch.device:
    if isinstance(device, int):
        device = torch.device("cuda", device)
    elif not isinstance(device, torch.device):
        device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("the NVLink collectives require a CUDA device")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def capture_id(stream: torch.cuda.Stream) -> int:
    """CUDA's id of the capture ``stream`` takes part in, 0 when not capturing."""
    try:
        from cuda.bindings import runtime as cudart
    except ImportError:  # pragma: no cover - cuda-python is in the image
        return 1 if torch.cuda.is_current_stream_capturing() else 0
    info = cudart.cudaStreamGetCaptureInfo(stream.cuda_stream)
    if info[0] != cudart.cudaError_t.cudaSuccess:
        return 0
    if info[1] != cudart.cudaStreamCaptureStatus.cudaStreamCaptureStatusActive:
        return 0
    return int(info[2])


def align_up(value: int, alignment: int) -> int:
    return (int(value) + alignment - 1) // alignment * alignment


def _env_int(name: str, default: int) -> int:
    raw = os.environ.get(name)
    return int(raw) if raw else default


class _StatusView:
    """Zero-copy view of the pinned status record (8 uint32 words per rank)."""

    WORDS = 8

    def __init__(self, address: int, records: int):
        self._words = (ctypes.c_uint32 * (self.WORDS * records)).from_address(address)

    def word(self, record: int, index: int) -> int:
        return int(self._words[record * self.WORDS + index])

    def set_word(self, record: int, index: int, value: int) -> None:
        self._words[record * self.WORDS + index] = value


# Rates measured on B200 that size the all-gather -> GEMM split between copy CTAs and
# GEMM CTAs: one CTA pushing 16-byte packs to a peer over NVLink sustains ~20 GB/s
# (benchmarks/microbench_nvlink.py, store, 4 packs in flight), and the tcgen05 GEMM
# sustains ~9 TFLOP/s per SM in bf16 (1354.8 TFLOP/s over 148 SMs) and ~10.7 in
# block-scaled fp8.
PUSH_GBS_PER_CTA = 20.0
FUSED_NORM_MAX_TOKENS = {1: 0, 2: 32, 8: 128}   # by world size; see NvlinkAllReduce.fused_norm_max_tokens
MIN_COPY_CTAS = 16        # fewer measured slower at TP2 and TP8 on every prefill shape
BF16_GEMM_TFLOPS_PER_SM = 9.0
FP8_GEMM_TFLOPS_PER_SM = 10.7


def copy_ctas_for(shard_bytes: int, world: int, flops: int, *, sms: int = 148,
                  gemm_tflops_per_sm: float = BF16_GEMM_TFLOPS_PER_SM, push_gbs_per_cta: float = PUSH_GBS_PER_CTA,
                  min_ctas: int = MIN_COPY_CTAS) -> int:
    """Copy CTAs for the fused all-gather -> GEMM so that pushing the shard to the
    ``world - 1`` peers takes about as long as the GEMM on the remaining SMs:
    c / (sms - c) = (bytes / push rate) / (flops / GEMM rate per SM).  Clamped to
    [min_ctas, sms / 2]; rank-invariant (shapes and world only)."""
    if world <= 1:
        return 0
    t_push = (world - 1) * shard_bytes / (push_gbs_per_cta * 1e9)       # seconds with one CTA
    t_gemm = flops / (gemm_tflops_per_sm * 1e12)                          # seconds with one SM
    c = sms * t_push / (t_push + t_gemm)
    return int(max(min_ctas, min(sms // 2, round(c))))


class NvlinkAllReduce:
    """One-shot / two-shot / NVLS collectives over NVLink symmetric memory."""

    algorithm = "nvlink"

    def __init__(
        self,
        *,
        exchange_group,
        device: torch.device | int | str,
        max_size: Optional[int] = None,
        max_gather_bytes: int = DEFAULT_MAX_GATHER_BYTES,
        threads: int = DEFAULT_THREADS,
        blocks: int = DEFAULT_BLOCKS,
        policy: Optional[CollectivePolicy] = None,
        enable_multicast: Optional[bool] = None,
        transport=None,
        pdl: Optional[bool] = None,
    ) -> None:
        self.device = normalize_device(device)
        self.rank = dist.get_rank(group=exchange_group)
        self.world_size = dist.get_world_size(group=exchange_group)
        self._group = exchange_group
        self._closed = False
        self._lock = threading.RLock()
        self._comm = None
        self._transport = None
        self._mc = (0, 0, 0)
        self._trace_map = None
        self._align_buffers: Optional[tuple[torch.Tensor, torch.Tensor]] = None
        self._gather_buffers: Optional[tuple[torch.Tensor, torch.Tensor]] = None
        self._prepared: set[torch.dtype] = set()
        self._stream_event = torch.cuda.Event()
        self._last_stream = None
        self._current_stream = None
        self._algo_cache: dict[tuple[int, torch.dtype], str] = {}  # the policy's choice per size
        self._algo_cache_policy = None
        self._capture_stream = None
        self._capture_id = 0
        self._calls = {"oneshot": 0, "twoshot": 0, "nvls": 0, "local": 0, "all_gather": 0, "reduce_scatter": 0,
                       "exchange": 0, "fused_norm": 0}
        # host-side accounting of issued collectives (a captured graph counts once, at capture)
        self._peer_bytes = 0      # bytes this rank sent to each peer over NVLink (P2P stores)
        self._nvls_bytes = 0      # bytes moved through the multicast alias
        if self.world_size not in SUPPORTED_WORLD_SIZES:
            raise ValueError(f"unsupported world size {self.world_size}; supported: {SUPPORTED_WORLD_SIZES}")
        if max_size is None:  # room for the measured dispatch ceiling of this world size
            max_size = max(DEFAULT_MAX_SIZE, default_dispatch_bytes(self.world_size))
        if int(max_size) < PACK_BYTES or int(max_size) % PACK_BYTES:
            raise ValueError("max_size must be a positive multiple of 16 bytes")
        if int(threads) % 32 or not 32 <= int(threads) <= 512:
            raise ValueError("threads must be a multiple of 32 between 32 and 512")
        if int(blocks) < 0:
            raise ValueError("blocks must be 0 (automatic) or positive")
        problems = removed_setting_problems(os.environ)
        if problems:
            raise ValueError("; ".join(problems))
        self.max_size = int(max_size)
        self.max_gather_bytes = int(max_gather_bytes)
        self.dispatch_max_bytes = _env_int(ENV_DISPATCH, min(self.max_size, default_dispatch_bytes(self.world_size)))
        if not PACK_BYTES <= self.dispatch_max_bytes <= self.max_size or self.dispatch_max_bytes % PACK_BYTES:
            raise ValueError("the dispatch limit must be 16-byte aligned and within the registered capacity")
        self.timeout_ms = checked_timeout_ms(_env_int(ENV_TIMEOUT_MS, DEFAULT_TIMEOUT_MS))
        self._threads = int(threads)
        self._blocks = int(blocks)
        if policy is None:
            env = dict(os.environ)
            crossover = dict(DEFAULT_ONESHOT_MAX)
            if env.get(ENV_CROSSOVER):
                import json

                crossover.update({int(k): int(v) for k, v in json.loads(env[ENV_CROSSOVER]).items()})
            policy = CollectivePolicy(self.dispatch_max_bytes, self.max_size, self.max_gather_bytes,
                                      oneshot_max_bytes=crossover,
                                      allow_nvls=env.get(ENV_NVLS, "0") not in ("", "0", "false", "False"),
                                      force=env.get(ENV_ALGO) or None)
        errors = policy.problems()
        if errors:
            raise ValueError("; ".join(errors))
        self.policy = policy
        self.topology = "nvswitch"
        want_mc = enable_multicast if enable_multicast is not None else policy.allow_nvls
        # capacities: one-shot holds a whole message, two-shot half a slot per chunk
        lam_cap = align_up(max(self.max_size, 2 * self.max_size // max(1, self.world_size) + 4096), 4096)
        ll_cap = align_up(min(LL_CAP, max(self.max_gather_bytes, PACK_BYTES)), 4096)
        push_cap = align_up(max(self.max_gather_bytes, PACK_BYTES), 4096)
        self._caps = (lam_cap, ll_cap, push_cap)
        mc_bytes = align_up(max(self.max_size, self.world_size * min(self.max_gather_bytes, self.max_size)),
                            4096) if (want_mc and self.world_size > 1) else 0

        C = _native.load()
        error: Optional[str] = None
        with torch.cuda.device(self.device):
            region_bytes = int(C.layout_total(self.world_size, *self._caps))
            config = {
                "api_version": API_VERSION, "abi": int(C.ABI_VERSION), "world_size": self.world_size,
                "max_size": self.max_size, "dispatch_max_bytes": self.dispatch_max_bytes,
                "max_gather_bytes": self.max_gather_bytes, "timeout_ms": self.timeout_ms,
                "threads": self._threads, "blocks": self._blocks, "caps": self._caps,
                "region_bytes": region_bytes, "multicast": bool(mc_bytes),
                "policy": (dict(policy.oneshot_max_bytes), policy.ll_max_bytes, policy.allow_nvls,
                           policy.nvls_min_bytes, policy.force),
                "sms": torch.cuda.get_device_properties(self.device).multi_processor_count,
            }
            statuses = symm.exchange(config, exchange_group)
            differing = [f"rank {i}: {sorted(k for k in config if s.get(k) != statuses[0].get(k))}"
                         for i, s in enumerate(statuses) if s != statuses[0]]
            if differing:
                raise RuntimeError("NVLink runtime setup failed: configuration differs from rank 0: "
                                   + "; ".join(differing))
            from ..transport import Geometry, NvlinkP2PTransport, NvlsTransport

            geometry = Geometry(self.world_size, self.rank, self.device.index, region_bytes, mc_bytes)
            factory = transport or (NvlsTransport if mc_bytes else NvlinkP2PTransport)
            self._transport = factory(geometry)
            self._transport.connect(exchange_group)
            self._transport.start()
            mc = self._transport.multicast()
            self._mc = mc or (0, 0, 0)
            try:
                self._comm = C.Comm(self.rank, self.world_size, self.device.index, *self._caps,
                                    self._transport.bases(), self._mc[0], self._mc[1], self._mc[2], False)
                self._comm.init_region()
                self._comm.set_timeout_us(1000 * self.timeout_ms)
            except Exception as exc:  # noqa: BLE001 - reported collectively
                error = str(exc)
            symm.collective_check(error, exchange_group, "NVLink runtime setup")
            dist.barrier(group=exchange_group)  # no peer pushes before every region is initialised
        self._status = _StatusView(self._comm.status_address(), 1)
        self.trace_path = None
        self._trace_map = None
        if trace.enabled():
            samples = C.clock_probe(self.device.index, 200)
            self.trace_path, self._trace_map, address = trace.open_trace(rank=self.rank, world=self.world_size,
                                                                         clock_samples=samples)
            self._comm.set_trace(address, trace.file_bytes())
            logger.info("collective trace %s", self.trace_path)
        self.has_multicast = bool(self._comm.has_multicast)
        self.set_pdl(os.environ.get(ENV_PDL, "1") != "0" if pdl is None else bool(pdl))
        if self.rank == 0:
            logger.info("NVLink collectives ready: world=%d region=%d MiB multicast=%s max_size=%d",
                        self.world_size, region_bytes >> 20, self.has_multicast, self.max_size)

    # -- construction ----------------------------------------------------------------
    @classmethod
    def from_exchange_group(cls, *, exchange_group, device, max_size: Optional[int] = None,
                            eager_buffer_bytes: Optional[int] = None,
                            max_gather_bytes: int = DEFAULT_MAX_GATHER_BYTES, threads: int = DEFAULT_THREADS,
                            blocks: int = DEFAULT_BLOCKS, **kwargs: Any) -> "NvlinkAllReduce":
        """Build the runtime collectively over ``exchange_group`` (a CPU/gloo group)."""
        if "kernels" in kwargs:
            raise TypeError("the kernels keyword is not supported: the kernels are compiled ahead of time")
        known = {k: kwargs[k] for k in ("policy", "enable_multicast", "transport", "pdl") if k in kwargs}
        capacity = None if max_size is None and not eager_buffer_bytes else \
            max(int(max_size or 0), int(eager_buffer_bytes or 0))
        return cls(exchange_group=exchange_group, device=device, max_size=capacity,
                   max_gather_bytes=max_gather_bytes, threads=threads, blocks=blocks, **known)

    @classmethod
    def from_process_group(cls, *, process_group, device, max_size: Optional[int] = None,
                           max_input_bytes: Optional[int] = None, **_ignored: Any) -> "NvlinkAllReduce":
        """Build the runtime with ``process_group`` as both the rank identity and the
        setup exchange (a CPU-capable group, e.g. gloo); further keywords are accepted
        and ignored, as in the reference (``sparknet/oneshot/runtime.py``)."""
        capacity = None if max_size is None and not max_input_bytes else \
            max(int(max_size or 0), int(max_input_bytes or 0))
        return cls(exchange_group=process_group, device=device, max_size=capacity)

    # -- policy --------------------------------------------------------------------------
    @property
    def supports_all_peer_auxiliary(self) -> bool:
        """True: the fused residual + RMSNorm epilogue is implemented."""
        return True

    def _live(self) -> None:
        if self._closed or self._comm is None:
            raise RuntimeError("NVLink runtime is closed")

    @staticmethod
    def _dtype_name(t: torch.Tensor) -> str:
        return str(t.dtype).replace("torch.", "")

    def should_allreduce(self, inp: torch.Tensor) -> bool:
        """Eligible below the jointly validated dispatch ceiling (rank-invariant)."""
        return self._accepts_allreduce(inp, self.dispatch_max_bytes)

    def _accepts_allreduce(self, inp: torch.Tensor, limit: int) -> bool:
        self._live()
        if inp.dtype not in SUPPORTED_DTYPES or not inp.is_cuda:
            return False
        if inp.device != self.device or not inp.is_contiguous():
            return False
        nbytes = inp.numel() * inp.element_size()
        return 0 < nbytes <= limit and nbytes % PACK_BYTES == 0

    def algorithm_for(self, nbytes: int, dtype: torch.dtype) -> str:
        """The all-reduce algorithm for ``nbytes`` of ``dtype`` (memoised per policy object)."""
        cache = getattr(self, "_algo_cache", None)
        if cache is None:
            return self._choose_algorithm(nbytes, dtype)
        if self._algo_cache_policy is not self.policy or len(cache) > 4096:
            cache.clear()
            self._algo_cache_policy = self.policy
        key = (int(nbytes), dtype)
        algo = cache.get(key)
        if algo is None:
            algo = cache[key] = self._choose_algorithm(nbytes, dtype)
        return algo

    def _choose_algorithm(self, nbytes: int, dtype: torch.dtype) -> str:
        algo = self.policy.all_reduce_backend(int(nbytes), str(dtype).replace("torch.", ""),
                                              world=self.world_size)
        if algo == "nccl":  # above dispatch but within capacity: the runtime still carries it
            algo = "oneshot" if nbytes <= self.policy.oneshot_limit(self.world_size) else "twoshot"
        if algo == "nvls" and not self.has_multicast:
            algo = "twoshot"  # rank-invariant: multicast availability was agreed collectively
        if self.world_size == 1:
            algo = "local"  # one rank: the sum is the input, one copy kernel
        return algo

    def prepare_channels(self, channel_ids: Sequence[str]) -> None:
        return None

    def for_stream(self, stream: object = None, *, channel_id: Optional[str] = None):
        return self

    def prepare(self, dtypes: Sequence[torch.dtype] = (torch.bfloat16,), *, padded_gather: bool = False) -> None:
        """Allocate scratch and warm every kernel outside any capture.

        Kernels are compiled ahead of time; preparing allocates the alignment
        scratch (and the padded-gather scratch with ``padded_gather=True``) and
        launches each dtype's kernels once collectively so first use inside a
        capture finds everything resident.
        """
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("preparation is refused inside a CUDA graph capture")
        for dtype in dtypes:
            if dtype not in SUPPORTED_DTYPES:
                raise ValueError(f"unsupported dtype {dtype}")
        with torch.cuda.device(self.device):
            self._aligned_scratch(0, torch.empty(PACK_BYTES, dtype=torch.uint8, device=self.device))
            if padded_gather:
                self._gather_scratch(PACK_BYTES)
            for dtype in dtypes:
                probe = torch.zeros(PACK_BYTES // torch.tensor([], dtype=dtype).element_size() * self.world_size,
                                    dtype=dtype, device=self.device)
                self.all_reduce(probe)
                self._prepared.add(dtype)
            torch.cuda.synchronize(self.device)
        self.check_health()

    # -- stream ordering -----------------------------------------------------------------
    # Collectives share the symmetric slots and the device epoch, so they run one at a
    # time.  On one stream that is the stream's own order; when a call arrives on another
    # stream, the new stream first waits for everything the previous one holds (the last
    # collective included).  The event is recorded only at such a switch, not per call.
    def _order_stream(self, capturing: bool) -> None:
        current = torch.cuda.current_stream(self.device)
        self._current_stream = current
        if capturing:
            cid = capture_id(current)
            if cid != self._capture_id:
                self._capture_id = cid
                self._capture_stream = current
            elif current != self._capture_stream:
                raise RuntimeError("NVLink collectives must all be captured on one stream")
            return
        last = self._last_stream
        if last is not None and current != last:
            self._stream_event.record(last)
            current.wait_event(self._stream_event)

    def _mark_stream(self, capturing: bool) -> None:
        if not capturing:
            self._last_stream = self._current_stream

    def _aligned_scratch(self, which: int, like: torch.Tensor) -> torch.Tensor:
        if self._align_buffers is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("alignment scratch must be allocated before capture; call prepare() first")
            raise_if_kernel_resolution_frozen("alignment scratch allocation", target=self)
            self._align_buffers = (torch.empty(self.max_size + PACK_BYTES, dtype=torch.uint8, device=self.device),
                                   torch.empty(self.max_size + PACK_BYTES, dtype=torch.uint8, device=self.device))
        nbytes = like.numel() * like.element_size()
        return self._align_buffers[which][:nbytes].view(like.dtype).view(like.shape)

    def _gather_scratch(self, padded: int) -> tuple[torch.Tensor, torch.Tensor]:
        if self._gather_buffers is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("gather scratch must be allocated before capture; call prepare(padded_gather=True)")
            raise_if_kernel_resolution_frozen("gather scratch allocation", target=self)
            capacity = align_up(self.max_gather_bytes, PACK_BYTES)
            self._gather_buffers = (torch.empty(capacity, dtype=torch.uint8, device=self.device),
                                    torch.empty(self.world_size * capacity, dtype=torch.uint8, device=self.device))
        staged, gathered = self._gather_buffers
        return staged[:padded], gathered[: self.world_size * padded]

    def _stream_ctx(self, stream):
        return torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()

    # -- all-reduce ------------------------------------------------------------------------
    def all_reduce(self, inp: torch.Tensor, *, out: Optional[torch.Tensor] = None, stream: object = None,
                   channel_id: Optional[str] = None, peer_input_ptrs: Optional[Sequence[int]] = None,
                   algorithm: Optional[str] = None) -> torch.Tensor:
        """Sum ``inp`` across ranks into ``out`` (allocated like ``inp`` when omitted).

        Executes any input within the registered capacity; which inputs to send here is
        the caller's (rank-invariant) decision, ``should_allreduce``.  ``algorithm``
        overrides the policy (benchmarks; must be the same on every rank).
        """
        del channel_id, peer_input_ptrs
        with self._lock:
            self.check_health()
            if not self._accepts_allreduce(inp, self.max_size):
                raise ValueError("input is not eligible for the NVLink all-reduce")
            if out is not None and (out.shape != inp.shape or out.dtype != inp.dtype or out.device != inp.device
                                    or not out.is_contiguous()):
                raise ValueError("out must be a contiguous tensor on the input's device matching the input")
            nbytes = inp.numel() * inp.element_size()
            algo = algorithm or self.algorithm_for(nbytes, inp.dtype)
            if algo not in ALGO_CODES or (algo == "local" and self.world_size != 1):
                raise ValueError(f"all-reduce algorithm {algo!r} is not available at world size {self.world_size}")
            with torch.cuda.device(self.device), self._stream_ctx(stream):
                capturing = torch.cuda.is_current_stream_capturing()
                if out is None:
                    out = torch.empty_like(inp)
                src = inp
                if inp.data_ptr() % PACK_BYTES:
                    src = self._aligned_scratch(0, inp)
                    src.copy_(inp)
                dst = out if out.data_ptr() % PACK_BYTES == 0 else self._aligned_scratch(1, out)
                self._order_stream(capturing)
                self._comm.all_reduce([src], [dst], ALGO_CODES[algo], self._threads, self._blocks)
                self._calls[algo] += 1
                self._account_reduce(algo, nbytes)
                if dst is not out:
                    out.copy_(dst)
                self._mark_stream(capturing)
        if not capturing:
            self.check_health()
        return out

    def all_reduce_residual_rmsnorm(self, inp: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
                                    eps: float = 1e-5, *, out: Optional[torch.Tensor] = None,
                                    residual_out: Optional[torch.Tensor] = None, stream: object = None,
                                    algorithm: Optional[str] = None, cluster: int = 8
                                    ) -> tuple[torch.Tensor, torch.Tensor]:
        """Fused ``residual += all_reduce(inp); out = rms_norm(residual) * gamma``.

        ``inp`` and ``residual`` are ``[tokens, hidden]``; returns ``(out, residual_out)``.
        One kernel up to :meth:`fused_norm_max_tokens` rows (bf16), the all-reduce then the
        add + RMSNorm kernel above it (or with ``algorithm`` forced, always one kernel).
        Rounds exactly where the unfused sequence would (after the all-reduce and after
        the add), so the new residual equals ``all_reduce(inp) + residual`` bit for bit,
        and every rank computes identical outputs.  ``residual_out`` may alias
        ``residual`` (in place, as vLLM's fused_add_rms_norm does).
        """
        with self._lock:
            self.check_health()
            self._live()
            if inp.dim() != 2 or residual.shape != inp.shape or gamma.shape != (inp.shape[1],):
                raise ValueError("fused norm takes inp/residual [tokens, hidden] and gamma [hidden]")
            if inp.dtype not in SUPPORTED_DTYPES or residual.dtype != inp.dtype or gamma.dtype != inp.dtype:
                raise ValueError("inp, residual and gamma must share a supported dtype")
            for t in (inp, residual, gamma):
                if not t.is_cuda or t.device != self.device or not t.is_contiguous() or t.data_ptr() % PACK_BYTES:
                    raise ValueError("fused norm tensors must be contiguous, 16-byte aligned, on the runtime device")
            tokens, hidden = inp.shape
            nbytes = inp.numel() * inp.element_size()
            if (algorithm is None and inp.dtype == torch.bfloat16 and tokens > self.fused_norm_max_tokens()
                    and self._accepts_allreduce(inp, self.max_size)):
                # more rows than the fused kernel wins at: the all-reduce, then the add +
                # RMSNorm kernel (the same residual bits; the output within one rounding)
                out = self.all_reduce(inp, out=out, stream=stream)
                residual_out = torch.empty_like(residual) if residual_out is None else residual_out
                with torch.cuda.device(self.device), self._stream_ctx(stream):
                    _native.load().add_rmsnorm(out, residual, residual_out, gamma, out, float(eps))
                return out, residual_out
            if algorithm is None:
                algorithm = self._fused_norm_algorithm(tokens, nbytes)
            with torch.cuda.device(self.device), self._stream_ctx(stream):
                capturing = torch.cuda.is_current_stream_capturing()
                out = torch.empty_like(inp) if out is None else out
                residual_out = torch.empty_like(residual) if residual_out is None else residual_out
                self._order_stream(capturing)
                self._comm.fused_norm([inp], [residual], gamma, float(eps), [out], [residual_out],
                                      ALGO_CODES[algorithm], cluster, 0)
                self._calls["fused_norm"] += 1
                self._account_reduce(algorithm, nbytes)
                self._mark_stream(capturing)
        if not capturing:
            self.check_health()
        return out, residual_out

    def fused_norm_max_tokens(self) -> int:
        """Most rows the single-kernel all-reduce + residual + RMSNorm carries; more go to
        the all-reduce then the add + RMSNorm kernel.  Measured with ``bench.py`` (256-call
        graphs, hidden 8192): on 8 B200s the fused kernel won up to 128 tokens (16.9 vs
        17.6 us) and lost at 256 (28.5 vs 22.8 us); on 2 it won up to 32 and lost at 128
        (14.5 vs 12.3 us); on one GPU the copy + add-norm pair was always faster."""
        table = FUSED_NORM_MAX_TOKENS
        smaller = [w for w in table if w <= self.world_size]
        return table[max(smaller)] if smaller else 0

    def _fused_norm_algorithm(self, tokens: int, nbytes: int) -> str:
        """One-shot or two-shot for the fused norm (rank-invariant: sizes and world)."""
        if self.world_size <= 2 or nbytes <= self.policy.oneshot_limit(self.world_size) or tokens < self.world_size:
            return "oneshot"
        return "twoshot"

    # -- fused prefill GEMMs (tcgen05) -------------------------------------------------------
    def _gemm_err(self) -> torch.Tensor:
        if getattr(self, "_gemm_err_word", None) is None:
            self._gemm_err_word = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._gemm_err_word

    def ag_gemm(self, x_shard: torch.Tensor, w: torch.Tensor, *, out: Optional[torch.Tensor] = None,
                copy_ctas: Optional[int] = None) -> torch.Tensor:
        """``all_gather(x_shard, dim=0) @ w.T`` in one kernel (sequence-parallel prefill).

        ``x_shard`` is this rank's ``[T/W, K]`` rows, ``w`` this rank's ``[N, K]``
        column shard (K-major).  Copy CTAs push the shard to every peer chunk by chunk
        while tcgen05 tiles consume own rows first and peers' rows as they land.  The
        number of copy CTAs defaults to :func:`copy_ctas_for` (push time balanced against
        GEMM time).
        """
        if copy_ctas is None:
            copy_ctas = copy_ctas_for(x_shard.numel() * x_shard.element_size(), self.world_size,
                                      2 * x_shard.shape[0] * self.world_size * x_shard.shape[1] * w.shape[0])
        with self._lock:
            self.check_health()
            self._live()
            capturing = torch.cuda.is_current_stream_capturing()
            with torch.cuda.device(self.device):
                if out is None:
                    out = torch.empty((x_shard.shape[0] * self.world_size, w.shape[0]), dtype=x_shard.dtype,
                                      device=self.device)
                self._order_stream(capturing)
                self._comm.ag_gemm(x_shard, w, out, self._gemm_err(), int(copy_ctas), 0)
                self._peer_bytes += x_shard.numel() * x_shard.element_size()
                self._mark_stream(capturing)
        return out

    def gemm_rs(self, a: torch.Tensor, w: torch.Tensor, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``reduce_scatter(a @ w.T, dim=0)`` in one kernel (row-parallel prefill GEMM).

        ``a`` is ``[T, K/W]`` (this rank's slice of the contraction), ``w`` is
        ``[N, K/W]``; returns this rank's ``[T/W, N]`` rows summed over ranks in fixed
        rank order from bf16 partials.
        """
        with self._lock:
            self.check_health()
            self._live()
            capturing = torch.cuda.is_current_stream_capturing()
            with torch.cuda.device(self.device):
                if out is None:
                    out = torch.empty((a.shape[0] // self.world_size, w.shape[0]), dtype=a.dtype, device=self.device)
                self._order_stream(capturing)
                self._comm.gemm_rs(a, w, out, self._gemm_err(), 0)
                self._peer_bytes += out.numel() * out.element_size()   # each owner's rows of the partial
                self._mark_stream(capturing)
        return out

    def ag_gemm_fp8(self, xq_shard: torch.Tensor, sfa_shard: torch.Tensor, w: torch.Tensor, sfw: torch.Tensor, *,
                    out: Optional[torch.Tensor] = None, copy_ctas: Optional[int] = None) -> torch.Tensor:
        """Block-scaled fp8 ``all_gather(x_shard) @ w.T`` in one kernel, bf16 out.

        ``xq_shard``/``sfa_shard`` and ``w``/``sfw`` come from
        ``sparknet.ops.fp8.quantize_act`` / ``quantize_weight`` (e4m3 with UE8M0 scales
        per 1 x 128 and 128 x 128).  The shard's rows and scales cross NVLink in fp8,
        half the bytes of the bf16 gather.
        """
        if copy_ctas is None:
            copy_ctas = copy_ctas_for(xq_shard.numel() + sfa_shard.numel(), self.world_size,
                                      2 * xq_shard.shape[0] * self.world_size * xq_shard.shape[1] * w.shape[0],
                                      gemm_tflops_per_sm=FP8_GEMM_TFLOPS_PER_SM)
        with self._lock:
            self.check_health()
            self._live()
            capturing = torch.cuda.is_current_stream_capturing()
            with torch.cuda.device(self.device):
                if out is None:
                    out = torch.empty((xq_shard.shape[0] * self.world_size, w.shape[0]), dtype=torch.bfloat16,
                                      device=self.device)
                self._order_stream(capturing)
                self._comm.ag_gemm_fp8(xq_shard, sfa_shard, w, sfw, out, self._gemm_err(), int(copy_ctas), 0)
                self._peer_bytes += xq_shard.numel() + sfa_shard.numel()
                self._mark_stream(capturing)
        return out

    def gemm_rs_fp8(self, aq: torch.Tensor, sfa: torch.Tensor, w: torch.Tensor, sfw: torch.Tensor, *,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Block-scaled fp8 ``reduce_scatter(a @ w.T)`` in one kernel; bf16 partials and
        output, summed in fixed rank order."""
        with self._lock:
            self.check_health()
            self._live()
            capturing = torch.cuda.is_current_stream_capturing()
            with torch.cuda.device(self.device):
                if out is None:
                    out = torch.empty((aq.shape[0] // self.world_size, w.shape[0]), dtype=torch.bfloat16,
                                      device=self.device)
                self._order_stream(capturing)
                self._comm.gemm_rs_fp8(aq, sfa, w, sfw, out, self._gemm_err(), 0)
                self._peer_bytes += out.numel() * out.element_size()
                self._mark_stream(capturing)
        return out

    def gemm_error(self) -> int:
        """The fused GEMMs' error word (0 = healthy; synchronises)."""
        return int(self._gemm_err().item())

    # -- health ------------------------------------------------------------------------------
    def set_timeout_ms(self, timeout_ms: int) -> None:
        """How long a wait may see nothing from a peer before the collective gives up.

        Kernels read the value from pinned memory when a wait first runs long, so it
        applies to captured graphs too.  Every rank should set the same value.
        """
        self.timeout_ms = checked_timeout_ms(timeout_ms)
        self._comm.set_timeout_us(1000 * self.timeout_ms)

    def set_pdl(self, enabled: bool) -> None:
        """Launch the collective kernels with programmatic dependent launch.

        Each collective is then scheduled while the previous kernel on its stream still
        runs; it waits (``griddepcontrol.wait``) until that kernel has finished before it
        reads its sequence number, and lets its own successor be scheduled once all of
        its blocks are running, so a chain of collectives (a graph) overlaps every
        launch with the previous call.  On by default (``SPARKNET_PDL=0`` turns it off):
        measured on B200 boxes (256-call graphs, geomean of 10 KiB-2 MiB), 6.35 -> 5.78 us
        at 2 ranks and 9.65 -> 8.98 us at 8 ranks.
        The one-rank copy always uses it.  Affects the calls issued after it, and graphs
        captured after it.
        """
        self._live()
        self._comm.set_pdl(bool(enabled))
        self.pdl = bool(self._comm.pdl)

    def failure(self) -> Optional[str]:
        """The failure report, or None while healthy (a pinned-memory read, no sync)."""
        if self._comm is None:
            return None
        seq = self._status.word(0, 1)
        if seq == 0:
            return None
        kind = FAIL_KINDS.get(self._status.word(0, 2), "failed")
        peer = self._status.word(0, 3)
        block = self._status.word(0, 4)
        waited = self._status.word(0, 5) / 1e6
        op = OP_NAMES.get(self._status.word(0, 6), "collective")
        return (f"NVLink {op} on rank {self.rank} {kind} waiting for rank {peer} (block {block}) after "
                f"{waited:.3f} s (timeout {self.timeout_ms / 1000:g} s) at sequence {seq}; the runtime is "
                "poisoned: every rank must call reset() or rebuild the group")

    def check_health(self) -> None:
        report = self.failure()
        if report is not None:
            raise RuntimeError(report)

    @property
    def poisoned(self) -> bool:
        return self.failure() is not None

    def reset(self) -> None:
        """Re-arm after a failure, collectively: every rank calls it with no collective in flight."""
        with self._lock:
            self._live()
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self._group)
            self._comm.init_region()
            dist.barrier(group=self._group)

    def barrier(self, blocks: int = 1) -> None:
        """A device-side barrier across ranks on the current stream (one kernel)."""
        with self._lock:
            self.check_health()
            capturing = torch.cuda.is_current_stream_capturing()
            with torch.cuda.device(self.device):
                self._order_stream(capturing)
                self._comm.barrier(int(blocks))
                self._mark_stream(capturing)

    # -- all-gather ------------------------------------------------------------------------------
    @staticmethod
    def _normalize_dim(inp: torch.Tensor, dim: int) -> int:
        return dim + inp.dim() if dim < 0 else dim

    def should_all_gather(self, inp: torch.Tensor, dim: int = -1, *, sliced: bool = False) -> bool:
        self._live()
        if not inp.is_cuda or inp.dim() == 0 or inp.device != self.device or not inp.is_contiguous():
            return False
        if inp.is_complex() or inp.is_sparse or inp.dtype == torch.bool:
            return False
        dim = self._normalize_dim(inp, dim)
        if dim not in (0, inp.dim() - 1):
            return False
        nbytes = inp.numel() * inp.element_size()
        if nbytes <= 0:
            return False
        if nbytes <= self.max_gather_bytes:
            return True
        if not sliced or torch.cuda.is_current_stream_capturing() or nbytes % PACK_BYTES:
            return False
        row_bytes = (inp.numel() // inp.shape[0]) * inp.element_size() if dim == 0 \
            else inp.shape[-1] * inp.element_size()
        return 0 < row_bytes <= self.max_gather_bytes and row_bytes % PACK_BYTES == 0

    def _direct_gather_layout(self, inp: torch.Tensor, dim: int) -> bool:
        nbytes = inp.numel() * inp.element_size()
        if nbytes % PACK_BYTES or inp.data_ptr() % PACK_BYTES:
            return False
        return dim == 0 or (inp.shape[-1] * inp.element_size()) % PACK_BYTES == 0

    def _gather_algorithm_fits(self, algo: str, shard_bytes: int) -> bool:
        if algo == "ll":
            return shard_bytes <= self._caps[1]
        if algo == "nvls":
            return self.has_multicast and shard_bytes * self.world_size <= self._mc[2]
        return algo == "push"

    def _launch_gather(self, src: torch.Tensor, dst: torch.Tensor, shard_bytes: int, row_bytes: int,
                       dst_row_stride: int, dst_src_stride: int, forced: Optional[str] = None) -> None:
        if forced is not None:
            if not self._gather_algorithm_fits(forced, shard_bytes):
                raise ValueError(f"all-gather algorithm {forced!r} cannot carry a {shard_bytes}-byte shard here")
            algo = forced
        else:
            algo = self.policy.all_gather_algorithm(shard_bytes, row_bytes=row_bytes or shard_bytes,
                                                    nvls_available=self.has_multicast)
            if algo == "ll" and shard_bytes > self._caps[1]:
                algo = "push"
            if algo == "nvls" and shard_bytes * self.world_size > self._mc[2]:
                algo = "push"
        self._comm.all_gather([src], [dst], shard_bytes, row_bytes, dst_row_stride, dst_src_stride,
                              GATHER_CODES[algo], self._threads, self._blocks)
        self._calls["all_gather"] += 1
        if algo == "nvls":
            self._nvls_bytes += shard_bytes
        else:
            self._peer_bytes += shard_bytes * (2 if algo == "ll" else 1)  # LL8 carries a flag per word

    def all_gather(self, inp: torch.Tensor, *, dim: int = -1, out: Optional[torch.Tensor] = None,
                   stream: object = None, sliced: bool = False, algorithm: Optional[str] = None) -> torch.Tensor:
        """Concatenate every rank's ``inp`` along ``dim`` (0 or the last dim).  ``algorithm``
        (``ll``, ``push`` or ``nvls``) overrides the policy's choice, as the probe's
        crossover sweep does; a choice that cannot carry the shard raises."""
        if algorithm is not None and algorithm not in GATHER_CODES:
            raise ValueError(f"all-gather algorithm must be one of {sorted(GATHER_CODES)}, got {algorithm!r}")
        with self._lock:
            self.check_health()
            if not self.should_all_gather(inp, dim, sliced=sliced):
                raise ValueError("input is not eligible for the NVLink all-gather")
            dim = self._normalize_dim(inp, dim)
            shape = list(inp.shape)
            shape[dim] *= self.world_size
            if out is not None and (list(out.shape) != shape or out.dtype != inp.dtype or out.device != inp.device
                                    or not out.is_contiguous()):
                raise ValueError("out must be a contiguous tensor on the input's device of the gathered shape")
            nbytes = inp.numel() * inp.element_size()
            with torch.cuda.device(self.device), self._stream_ctx(stream):
                capturing = torch.cuda.is_current_stream_capturing()
                if nbytes > self.max_gather_bytes:
                    if algorithm not in (None, "push"):
                        raise ValueError(f"a {nbytes}-byte shard is gathered in slices by the push kernel; "
                                         f"{algorithm!r} cannot carry it")
                    out = torch.empty(shape, dtype=inp.dtype, device=inp.device) if out is None else out
                    self._order_stream(capturing)
                    self._sliced_gather(inp, out, dim)
                    self._mark_stream(capturing)
                    return out
                direct = self._direct_gather_layout(inp, dim) and (out is None or out.data_ptr() % PACK_BYTES == 0)
                if direct:
                    out = torch.empty(shape, dtype=inp.dtype, device=inp.device) if out is None else out
                    if dim == 0:
                        row, row_stride, src_stride = 0, 0, nbytes
                    else:
                        row = inp.shape[-1] * inp.element_size()
                        row_stride, src_stride = row * self.world_size, row
                    self._order_stream(capturing)
                    self._launch_gather(inp, out, nbytes, row, row_stride, src_stride, forced=algorithm)
                    self._mark_stream(capturing)
                    result = out
                else:
                    padded = align_up(nbytes, PACK_BYTES)
                    staged, gathered = self._gather_scratch(padded)
                    staged[:nbytes].copy_(inp.reshape(-1).view(torch.uint8))
                    self._order_stream(capturing)
                    self._launch_gather(staged, gathered, padded, 0, 0, padded, forced=algorithm)
                    self._mark_stream(capturing)
                    stacked = (gathered.view(self.world_size, padded)[:, :nbytes].reshape(-1).view(inp.dtype)
                               .reshape(self.world_size, *inp.shape))
                    result = stacked.movedim(0, dim).reshape(shape)
                    if out is None:
                        result = result.contiguous()
                    else:
                        out.copy_(result)
                        result = out
        if not capturing:
            self.check_health()
        return result

    def _sliced_gather(self, inp: torch.Tensor, out: torch.Tensor, dim: int) -> None:
        nbytes = inp.numel() * inp.element_size()
        if dim == 0:
            rows = inp.shape[0]
            row_bytes = nbytes // rows
            max_rows = max(1, self.max_gather_bytes // row_bytes)
            flat_in = inp.reshape(rows, -1)
            out_rows = out.reshape(self.world_size * rows, -1)
            for lo in range(0, rows, max_rows):
                hi = min(rows, lo + max_rows)
                # shard slice lo:hi of every source lands at rows src*rows + lo
                self._comm.all_gather([flat_in[lo:hi]], [out_rows[lo:]], (hi - lo) * row_bytes, 0, 0, nbytes,
                                      GATHER_CODES["push"], self._threads, self._blocks)
                if not torch.cuda.is_current_stream_capturing():
                    self.check_health()
        else:
            width = inp.shape[-1]
            rows = inp.numel() // width
            row_bytes = width * inp.element_size()
            max_rows = max(1, self.max_gather_bytes // row_bytes)
            inp2 = inp.reshape(rows, width)
            out2 = out.reshape(rows, self.world_size * width)
            for lo in range(0, rows, max_rows):
                hi = min(rows, lo + max_rows)
                self._comm.all_gather([inp2[lo:hi]], [out2[lo:hi]], (hi - lo) * row_bytes, row_bytes,
                                      row_bytes * self.world_size, row_bytes, GATHER_CODES["push"],
                                      self._threads, self._blocks)
                if not torch.cuda.is_current_stream_capturing():
                    self.check_health()

    # -- reduce-scatter ----------------------------------------------------------------------------
    def should_reduce_scatter(self, inp: torch.Tensor, dim: int = 0) -> bool:
        self._live()
        if inp.dtype not in SUPPORTED_DTYPES or not inp.is_cuda or inp.dim() == 0:
            return False
        if inp.device != self.device or not inp.is_contiguous():
            return False
        if self._normalize_dim(inp, dim) != 0 or inp.shape[0] % self.world_size:
            return False
        nbytes = inp.numel() * inp.element_size()
        chunk = nbytes // self.world_size
        if chunk <= 0 or chunk % PACK_BYTES:
            return False
        if chunk <= self._caps[0]:
            return True
        if torch.cuda.is_current_stream_capturing():
            return False
        row_bytes = chunk // (inp.shape[0] // self.world_size)
        return row_bytes % PACK_BYTES == 0 and row_bytes <= self._caps[0]

    def reduce_scatter(self, inp: torch.Tensor, *, dim: int = 0, out: Optional[torch.Tensor] = None,
                       stream: object = None) -> torch.Tensor:
        """Reduce-scatter along dim 0 in fixed rank order with fp32 accumulation."""
        with self._lock:
            self.check_health()
            if not self.should_reduce_scatter(inp, dim):
                raise ValueError("input is not eligible for the NVLink reduce-scatter")
            local_rows = inp.shape[0] // self.world_size
            out_shape = (local_rows, *inp.shape[1:])
            if out is not None and (tuple(out.shape) != out_shape or out.dtype != inp.dtype
                                    or out.device != inp.device or not out.is_contiguous()):
                raise ValueError("out must be a contiguous tensor on the input's device of the scattered shape")
            nbytes = inp.numel() * inp.element_size()
            chunk = nbytes // self.world_size
            with torch.cuda.device(self.device), self._stream_ctx(stream):
                capturing = torch.cuda.is_current_stream_capturing()
                out = torch.empty(out_shape, dtype=inp.dtype, device=inp.device) if out is None else out
                src = inp
                if inp.data_ptr() % PACK_BYTES:
                    src = self._aligned_scratch(0, inp) if nbytes <= self.max_size else inp.clone()
                    src.copy_(inp)
                dst = out if out.data_ptr() % PACK_BYTES == 0 else torch.empty_like(out)
                self._order_stream(capturing)
                if chunk <= self._caps[0]:
                    self._comm.reduce_scatter([src], [dst], chunk, chunk, self._threads, self._blocks)
                else:
                    row_bytes = chunk // local_rows
                    max_rows = max(1, self._caps[0] // row_bytes)
                    src_rows = src.reshape(inp.shape[0], -1)
                    dst_rows = dst.reshape(local_rows, -1)
                    for lo in range(0, local_rows, max_rows):
                        hi = min(local_rows, lo + max_rows)
                        self._comm.reduce_scatter([src_rows[lo:]], [dst_rows[lo:hi]], (hi - lo) * row_bytes, chunk,
                                                  self._threads, self._blocks)
                        if not capturing:
                            self.check_health()
                self._calls["reduce_scatter"] += 1
                self._peer_bytes += chunk
                if dst is not out:
                    out.copy_(dst)
                self._mark_stream(capturing)
        if not capturing:
            self.check_health()
        return out

    # -- exchange / all-to-all -------------------------------------------------------------------
    def should_exchange(self, chunks: torch.Tensor, parts: Optional[torch.Tensor] = None) -> bool:
        self._live()
        if not chunks.is_cuda or chunks.device != self.device or chunks.dim() < 2:
            return False
        if chunks.is_complex() or chunks.is_sparse or chunks.dtype == torch.bool:
            return False
        if chunks.shape[0] != self.world_size or not chunks[0].is_contiguous():
            return False
        elem = chunks.element_size()
        chunk_bytes = chunks[0].numel() * elem
        if chunk_bytes == 0:
            return True
        if chunk_bytes % PACK_BYTES or (chunks.stride(0) * elem) % PACK_BYTES or chunks.data_ptr() % PACK_BYTES:
            return False
        if parts is not None:
            if (not parts.is_cuda or parts.device != self.device or parts.shape != chunks.shape
                    or parts.dtype != chunks.dtype or not parts[0].is_contiguous()):
                return False
            if (parts.stride(0) * elem) % PACK_BYTES or parts.data_ptr() % PACK_BYTES:
                return False
        if chunk_bytes <= self._caps[2]:
            return True
        if torch.cuda.is_current_stream_capturing():
            return False
        row_bytes = chunk_bytes // chunks.shape[1]
        return row_bytes % PACK_BYTES == 0 and row_bytes <= self._caps[2]

    def exchange(self, chunks: torch.Tensor, parts: Optional[torch.Tensor] = None, *,
                 out: Optional[torch.Tensor] = None, copy_self: bool = False, stream: object = None) -> torch.Tensor:
        """Send ``chunks[p]`` to peer ``p``; receive peer ``p``'s chunk into ``parts[p]``."""
        if parts is None and out is not None:
            parts = out
        with self._lock:
            self.check_health()
            if not self.should_exchange(chunks, parts):
                raise ValueError("input is not eligible for the NVLink exchange")
            parts = torch.empty(chunks.shape, dtype=chunks.dtype, device=chunks.device) if parts is None else parts
            elem = chunks.element_size()
            chunk_bytes = chunks[0].numel() * elem
            if chunk_bytes == 0:
                return parts
            src_stride = chunks.stride(0) * elem
            dst_stride = parts.stride(0) * elem
            with torch.cuda.device(self.device), self._stream_ctx(stream):
                capturing = torch.cuda.is_current_stream_capturing()
                self._order_stream(capturing)
                if chunk_bytes <= self._caps[2]:
                    self._launch_exchange(chunks, parts, chunk_bytes, src_stride, dst_stride, 0, -1, copy_self)
                else:
                    rows = chunks.shape[1]
                    row_bytes = chunk_bytes // rows
                    max_rows = max(1, self._caps[2] // row_bytes)
                    for lo in range(0, rows, max_rows):
                        hi = min(rows, lo + max_rows)
                        self._launch_exchange(chunks[:, lo:hi], parts[:, lo:hi], (hi - lo) * row_bytes, src_stride,
                                              dst_stride, 0, -1, copy_self)
                        if not capturing:
                            self.check_health()
                self._mark_stream(capturing)
        if not capturing:
            self.check_health()
        return parts

    def _launch_exchange(self, src: torch.Tensor, dst: torch.Tensor, chunk_bytes: int, src_stride: int,
                         dst_stride: int, total_src_bytes: int, valid_out_bytes: int, copy_self: bool) -> None:
        # the kernel addresses chunks by byte strides from the first element
        self._comm.exchange([src], [dst], chunk_bytes, src_stride, dst_stride, total_src_bytes,
                            valid_out_bytes, bool(copy_self), self._threads, self._blocks)
        self._calls["exchange"] += 1
        self._peer_bytes += chunk_bytes

    def should_all_to_all_rows(self, inp: torch.Tensor, rows: int) -> bool:
        self._live()
        if not inp.is_cuda or inp.device != self.device or inp.dim() < 1 or not inp.is_contiguous():
            return False
        if inp.is_complex() or inp.is_sparse or inp.dtype == torch.bool:
            return False
        total, rows = int(inp.shape[0]), int(rows)
        if rows <= 0 or total <= 0 or total > self.world_size * rows or inp.data_ptr() % PACK_BYTES:
            return False
        row_bytes = (inp.numel() // total) * inp.element_size()
        if row_bytes <= 0 or row_bytes % PACK_BYTES:
            return False
        if rows * row_bytes <= self._caps[2]:
            return True
        if torch.cuda.is_current_stream_capturing():
            return False
        return row_bytes <= self._caps[2]

    def all_to_all_rows(self, inp: torch.Tensor, rows: int, *, out: Optional[torch.Tensor] = None,
                        stream: object = None) -> torch.Tensor:
        """Exchange ``rows``-row blocks of ``inp`` into ``(world_size, rows, *inp.shape[1:])``.

        Rows at or beyond ``inp.shape[0]`` (the same count on every rank) do not exist;
        only the first ``min(rows, total - rank * rows)`` rows of each received block
        are written.
        """
        with self._lock:
            self.check_health()
            if not self.should_all_to_all_rows(inp, rows):
                raise ValueError("input is not eligible for the NVLink all_to_all_rows")
            rows, total = int(rows), int(inp.shape[0])
            out_shape = (self.world_size, rows, *inp.shape[1:])
            if out is not None and (tuple(out.shape) != out_shape or out.dtype != inp.dtype
                                    or out.device != inp.device or not out.is_contiguous()
                                    or out.data_ptr() % PACK_BYTES):
                raise ValueError("out must be a 16-byte-aligned contiguous tensor of shape (world_size, rows, ...)")
            row_bytes = (inp.numel() // total) * inp.element_size()
            chunk_bytes = rows * row_bytes
            with torch.cuda.device(self.device), self._stream_ctx(stream):
                capturing = torch.cuda.is_current_stream_capturing()
                out = inp.new_empty(out_shape) if out is None else out
                self._order_stream(capturing)
                max_rows = max(1, self._caps[2] // row_bytes)
                flat = inp.reshape(total, -1)
                for lo in range(0, rows, max_rows):
                    hi = min(rows, lo + max_rows)
                    slice_rows = hi - lo
                    own = max(0, min(slice_rows, total - (self.rank * rows + lo)))
                    src_total = max(0, total - lo) * row_bytes
                    src = flat[lo:] if lo < total else flat[:1]
                    self._comm.exchange([src], [out[:, lo:hi]], slice_rows * row_bytes, chunk_bytes,
                                        chunk_bytes, src_total, own * row_bytes, True, self._threads, self._blocks)
                    self._calls["exchange"] += 1
                    if not capturing and hi < rows:
                        self.check_health()
                self._mark_stream(capturing)
        if not capturing:
            self.check_health()
        return out

    # -- capture / diagnostics / lifecycle -----------------------------------------------------
    def _forget_stream_order(self) -> None:
        """Drop the remembered launch stream and capture identity (see ``capture``)."""
        self._last_stream, self._capture_stream, self._capture_id = None, None, 0

    @contextmanager
    def capture(self, stream: object = None, *, channel_id: Optional[str] = None):
        """Scope for CUDA-graph capture of NVLink collectives.

        Captured collectives read their sequence number from the device-resident epoch
        at replay time, so nothing host-side is baked into the graph.  What the runtime
        forgets on entry and on exit is its stream ordering: an event recorded outside a
        capture may not be waited on inside one, and one recorded inside belongs to the
        graph.  Within the scope every collective uses one stream.  ``stream`` and
        ``channel_id`` are accepted for the reference's signature; the stream in use is
        the one the first captured collective runs on."""
        del stream, channel_id
        self._forget_stream_order()
        try:
            yield self
        finally:
            self._forget_stream_order()

    def _account_reduce(self, algo: str, nbytes: int) -> None:
        if algo == "oneshot":
            self._peer_bytes += nbytes
        elif algo == "twoshot":
            self._peer_bytes += 2 * nbytes // max(1, self.world_size)
        elif algo == "nvls":
            self._nvls_bytes += nbytes

    def stats(self) -> dict[str, Any]:
        lam, ll, push = self._caps
        info: dict[str, Any] = {
            "world_size": self.world_size, "rank": self.rank, "topology": self.topology,
            "transport": "nvlink-p2p" + ("+nvls" if self.has_multicast else ""),
            "max_size": self.max_size, "dispatch_max_bytes": self.dispatch_max_bytes,
            "max_gather_bytes": self.max_gather_bytes, "lamport_slot_bytes": lam, "ll_slot_bytes": ll,
            "push_slot_bytes": push, "timeout_ms": self.timeout_ms, "pdl": getattr(self, "pdl", False),
            "threads": self._threads,
            "blocks": self._blocks, "multicast": self.has_multicast,
            "calls": dict(self._calls), "ops_posted": sum(self._calls.values()),
            "bytes_pushed_per_peer": self._peer_bytes, "nvls_bytes": self._nvls_bytes,
            "nvls_ops": self._calls.get("nvls", 0),
            "oneshot_max_bytes": self.policy.oneshot_limit(self.world_size),
        }
        if self._comm is not None:
            info["status"] = dict(self._comm.status(0))
            info["error_seq"] = info["status"]["failed_seq"]
            if not torch.cuda.is_current_stream_capturing():
                ctrl = dict(self._comm.ctrl(0))
                info.update({"epoch": ctrl["epoch"], "device_ops": ctrl["ops"], "poison": ctrl["poison"]})
        return info

    def close(self) -> None:
        """Release this rank's regions (collective: every rank closes, none keeps using
        the group).  The device is drained first, so no kernel of this rank is still
        reading or writing a peer's region when the mappings go; the trace file stays on
        disk for collection, only its mapping is dropped."""
        with self._lock:
            if self._closed:
                return
            self._closed = True
            comm, transport, trace = self._comm, self._transport, self._trace_map
            self._comm, self._transport, self._trace_map = None, None, None
            try:
                torch.cuda.synchronize(self.device)
            except Exception:  # noqa: BLE001 - a failed device still releases its mappings
                logger.debug("device drain before close failed", exc_info=True)
            if comm is not None and trace is not None:
                with contextlib.suppress(Exception):
                    comm.set_trace(0, 0)  # stop stamping before the mapping goes
                    trace.flush()
            if transport is not None:
                transport.stop()
                transport.close()

    def __del__(self) -> None:  # pragma: no cover - defensive teardown
        # no module globals here: at interpreter exit they may already be gone
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


__all__ = ["API_VERSION", "DEFAULT_MAX_GATHER_BYTES", "DEFAULT_MAX_SIZE", "SUPPORTED_DTYPES",
           "SUPPORTED_WORLD_SIZES", "TOPOLOGIES", "NvlinkAllReduce", "discover_hcas", "discover_nvlink_gpus",
           "is_supported"]
