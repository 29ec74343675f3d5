#!/usr/bin/env python3
"""Model-free qualification of the collective policy on one NVSwitch box.

Run one rank per GPU (``torch.distributed.run --nproc-per-node N -m
sparknet.probe.collectives``, or ``sparknet probe render-command`` for the bounded
container).  The probe initialises torch.distributed, builds the NVLink runtime from
the environment a recipe sets (or the default policy), then checks the policy
exactly: eligible all-reduces and all-gathers through the NVLink kernels, the rest
through NCCL; bf16/fp32, tiny, unaligned and large messages, both sides of every
limit, eager and graph-replayed with changing inputs.  With ``--benchmark`` it times
steady graph-replayed latency per (operation, size) as the median over samples of
the slowest rank, with NVLink counters around the timed cases; ``--sweep`` adds
every algorithm (one-shot, two-shot, NVLS, NCCL) for the crossover table.

Reference behaviour: ``sparknet/probe/collectives.py:33-309`` (2-4 RoCE ranks); this
probe runs 1, 2, 4 or 8 GPUs.  A passing probe is a prerequisite for serving, not
serving acceptance.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import sys
from contextlib import contextmanager, nullcontext
from dataclasses import dataclass
from datetime import timedelta


def _policy_from_environment():
    from sparknet.policy import NVLINK_POLICY, CollectivePolicy

    env = dict(os.environ)
    if env.get("SPARKNET_ALLREDUCE_CAPACITY_BYTES") and env.get("SPARKNET_ALLGATHER_MAX_BYTES"):
        return CollectivePolicy.from_environment(env)
    return NVLINK_POLICY


@dataclass(frozen=True)
class Route:
    """Where one probe collective went: ``backend`` is ``nccl`` or the NVLink algorithm
    (``oneshot``, ``twoshot``, ``nvls``, ``local``) the runtime ran."""

    operation: str
    backend: str
    nbytes: int

    @property
    def nvlink(self) -> bool:
        return self.backend != "nccl"


class PolicyCommunicator:
    """The probe's dispatcher: the explicit policy over NCCL and the NVLink runtime.

    Every call is routed by ``route()``: the policy names a backend from the operation,
    dtype, size and world (rank-invariant), and for an NVLink backend the runtime's own
    eligibility must agree, otherwise the probe fails instead of quietly using NCCL.
    Each route is tallied in ``ledger`` (``(operation, backend) -> [calls, bytes]``) so
    that ``check_runtime_counters`` can hold the runtime's counters to the routing.
    The reference's probe dispatcher (``sparknet/probe/collectives.py:33-89`` there)
    has the same public methods over its RoCE runtime; this one adds the forced arms
    of the crossover sweep and the ledger.
    """

    def __init__(self, runtime, policy, device, world_size):
        import torch
        import torch.distributed as dist

        self._torch, self._dist = torch, dist
        self.runtime, self.policy, self.device, self.world_size = runtime, policy, device, world_size
        self.ledger: dict[tuple[str, str], list[int]] = {}
        self.last_route: Route | None = None

    # -- routing -------------------------------------------------------------------
    def route(self, operation: str, tensor, *, dim: int = 0, forced: str | None = None) -> Route:
        nbytes = tensor.numel() * tensor.element_size()
        dtype = str(tensor.dtype).rsplit(".", 1)[-1]
        if forced is not None:
            backend = forced
        elif self.runtime is None:
            backend = "nccl"
        elif operation == "all_reduce":
            backend = self.policy.all_reduce_backend(nbytes, dtype, contiguous=tensor.is_contiguous(),
                                                     world=self.world_size)
            if backend != "nccl" and not self.runtime.should_allreduce(tensor):
                raise RuntimeError(f"all-reduce of {nbytes} bytes: the policy chose {backend}, the runtime "
                                   "refuses the tensor (policy and runtime eligibility disagree)")
            if backend != "nccl":
                backend = self.runtime.algorithm_for(nbytes, tensor.dtype)
        elif operation == "all_gather":
            backend = self.policy.all_gather_backend(nbytes, dtype, dim=dim, ndim=tensor.dim(),
                                                     contiguous=tensor.is_contiguous())
            if backend != "nccl" and not self.runtime.should_all_gather(tensor, dim):
                raise RuntimeError(f"all-gather of {nbytes} bytes: the policy chose the NVLink kernel, the "
                                   "runtime refuses the tensor (policy and runtime eligibility disagree)")
        elif operation == "reduce_scatter":
            within = self.policy.reduce_scatter_backend(nbytes, self.policy.all_reduce_capacity_bytes) != "nccl"
            backend = "oneshot" if within and self.runtime.should_reduce_scatter(tensor) else "nccl"
        else:
            raise ValueError(f"unknown probe operation {operation!r}")
        tally = self.ledger.setdefault((operation, backend), [0, 0])
        tally[0] += 1
        tally[1] += nbytes
        self.last_route = Route(operation, backend, nbytes)
        return self.last_route

    def backend_for_all_reduce(self, tensor) -> str:
        """The backend the policy picks for this tensor (no call is made or tallied)."""
        if self.runtime is None:
            return "nccl"
        nbytes = tensor.numel() * tensor.element_size()
        return self.policy.all_reduce_backend(nbytes, str(tensor.dtype).rsplit(".", 1)[-1],
                                              contiguous=tensor.is_contiguous(), world=self.world_size)

    # -- collectives -----------------------------------------------------------------
    def all_reduce(self, tensor, *, algorithm: str | None = None):
        r = self.route("all_reduce", tensor, forced=algorithm)
        if r.nvlink:
            return self.runtime.all_reduce(tensor, algorithm=r.backend)
        result = tensor.clone()
        self._dist.all_reduce(result)
        return result

    def all_gather(self, tensor, dim=0, *, force_nccl: bool = False, algorithm: str | None = None):
        """``algorithm`` (``ll``, ``push`` or ``nvls``) forces the NVLink kernel's protocol
        (the crossover sweep's arms); ``force_nccl`` forces NCCL."""
        r = self.route("all_gather", tensor, dim=dim, forced="nccl" if force_nccl else algorithm)
        if r.nvlink:
            return self.runtime.all_gather(tensor, dim=dim, algorithm=algorithm)
        pieces = [self._torch.empty_like(tensor) for _ in range(self.world_size)]
        self._dist.all_gather(pieces, tensor.contiguous())
        return self._torch.cat(pieces, dim=dim)

    def reduce_scatter(self, tensor, dim=0, *, force_nccl: bool = False):
        if dim != 0:
            raise ValueError("the probe reduce-scatters along dim 0 only")
        r = self.route("reduce_scatter", tensor, forced="nccl" if force_nccl else None)
        if r.nvlink:
            return self.runtime.reduce_scatter(tensor)
        shape = (tensor.shape[0] // self.world_size, *tensor.shape[1:])
        result = self._torch.empty(shape, dtype=tensor.dtype, device=tensor.device)
        self._dist.reduce_scatter_tensor(result, tensor.contiguous())
        return result


# runtime call counter that moves for one NVLink route of each operation
_RUNTIME_COUNTER = {"all_gather": "all_gather", "reduce_scatter": "reduce_scatter"}


def runtime_calls_expected(ledger_delta: dict[tuple[str, str], int]) -> dict[str, int]:
    """The runtime ``stats()['calls']`` increments that the routed calls imply: an
    all-reduce counts under its algorithm, the other operations under their name;
    NCCL routes move no runtime counter."""
    want: dict[str, int] = {}
    for (operation, backend), calls in ledger_delta.items():
        if backend == "nccl" or not calls:
            continue
        key = backend if operation == "all_reduce" else _RUNTIME_COUNTER[operation]
        want[key] = want.get(key, 0) + calls
    return want


def check_runtime_counters(before_calls: dict, after_calls: dict, ledger_before: dict, ledger_after: dict,
                           *, what: str, graph_replays: int = 0, calls_per_graph: int = 0) -> dict[str, int]:
    """Raise unless the runtime's call counters moved exactly as the routing says.

    Counters move when a call is issued (eagerly or while captured), not on replay, so
    ``graph_replays`` only matters for the byte estimate the caller derives."""
    ledger_delta = {k: ledger_after.get(k, [0, 0])[0] - ledger_before.get(k, [0, 0])[0]
                    for k in set(ledger_after) | set(ledger_before)}
    want = runtime_calls_expected(ledger_delta)
    moved = {k: after_calls.get(k, 0) - before_calls.get(k, 0) for k in set(after_calls) | set(before_calls)}
    moved = {k: v for k, v in moved.items() if v}
    if moved != want:
        raise RuntimeError(f"{what}: runtime counters moved {moved}, the policy's routing implies {want}")
    return want


def nvlink_bytes_expected(route: Route, world: int) -> int:
    """Bytes this rank must send over NVLink for one call on ``route`` (0 for NCCL and
    for one rank): one-shot pushes the whole message to every peer, two-shot 2(W-1)/W
    of it, the all-gather its shard to every peer, the reduce-scatter (W-1)/W."""
    if not route.nvlink or world < 2:
        return 0
    n, peers = route.nbytes, world - 1
    if route.operation == "all_reduce":
        if route.backend == "oneshot":
            return n * peers
        if route.backend in ("twoshot", "nvls"):
            return 2 * n * peers // world
        return 0
    if route.operation == "all_gather":
        return n if route.backend == "nvls" else n * peers  # NVLS: one copy, the switch fans it out
    return n * peers // world


@contextmanager
def reporting_failure(runtime):
    """Turn an exception raised after a failed NVLink collective into the runtime's own
    failure report (which rank was waited for, in which op), chained to the original.
    Exceptions with no collective failure behind them pass through unchanged."""
    try:
        yield
    except Exception as error:
        diagnosis = None if runtime is None else runtime.failure()
        if diagnosis is None:
            raise
        raise RuntimeError(diagnosis) from error


def _init(args):
    import torch
    import torch.distributed as dist

    if "RANK" in os.environ and args.rank is None:
        rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
        local = int(os.environ.get("LOCAL_RANK", rank))
        init = "env://"
    else:
        if args.rank is None or args.world_size is None or args.master_addr is None:
            raise SystemExit("run under torch.distributed.run, or pass --rank --world-size --master-addr")
        rank, world, local = args.rank, args.world_size, args.local_rank if args.local_rank is not None else 0
        init = f"tcp://{args.master_addr}:{args.master_port}"
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group(backend="cpu:gloo,cuda:nccl", world_size=world, rank=rank, init_method=init,
                            timeout=timedelta(seconds=120), device_id=device)
    return rank, world, device, dist.new_group(backend="gloo", timeout=timedelta(seconds=120))


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--rank", type=int, default=None)
    parser.add_argument("--local-rank", type=int, default=None)
    parser.add_argument("--world-size", type=int, choices=(1, 2, 4, 8), default=None)
    parser.add_argument("--master-addr", default=None)
    parser.add_argument("--master-port", type=int, default=29650)
    from sparknet.topology.gpumap import TRANSPORTS, uses_oneshot

    parser.add_argument("--transport", choices=TRANSPORTS, default=os.environ.get("SPARKNET_TRANSPORT", "nvlink"))
    parser.add_argument("--benchmark", action="store_true", help="after correctness, time steady graph latency")
    parser.add_argument("--sweep", action="store_true", help="benchmark every algorithm (one-shot/two-shot/NVLS/NCCL)")
    parser.add_argument("--counter-samples", action="store_true", help="NVLink counter deltas around each case")
    # 1, 6, 48 and 96 tokens of a 5,120-wide residual and 2 MiB (the reference's decode shapes), bf16 elements
    parser.add_argument("--lengths", type=int, nargs="+", default=[5120, 30720, 245760, 491520, 1048576])
    parser.add_argument("--dtypes", nargs="+", default=["bfloat16", "float32"])
    parser.add_argument("--operations", nargs="+", default=["all_reduce", "all_gather", "reduce_scatter"])
    parser.add_argument("--numerics", action="store_true", help="cancellation-sensitive reduction-order fingerprints")
    parser.add_argument("--skip-correctness", action="store_true")
    parser.add_argument("--output", default="", help="write the JSON result here as well as to stdout")
    parser.add_argument("--runtime-threads", type=int, default=None)
    parser.add_argument("--runtime-blocks", type=int, default=None)
    parser.add_argument("--pdl", action="store_true",
                        help="launch the NVLink collectives with programmatic dependent launch")
    args = parser.parse_args(argv)
    if any(n < 8 or n > (64 << 20) or n % 8 for n in args.lengths):
        parser.error("lengths must be multiples of 8 elements between 8 and 64 Mi")

    import torch
    import torch.distributed as dist

    from sparknet.probe import counters as nvcounters

    rank, world, device, cpu_group = _init(args)
    runtime, policy = None, None
    if uses_oneshot(args.transport):
        from sparknet import oneshot

        policy = _policy_from_environment()
        geometry = {k: v for k, v in (("threads", args.runtime_threads), ("blocks", args.runtime_blocks))
                    if v is not None}
        runtime = oneshot.AllReduce.from_exchange_group(
            exchange_group=cpu_group, device=device, max_size=policy.all_reduce_capacity_bytes,
            max_gather_bytes=policy.all_gather_shard_bytes, policy=policy,
            enable_multicast=(args.transport == "nvlink-nvls" or policy.allow_nvls), **geometry)
        if runtime.dispatch_max_bytes != policy.all_reduce_dispatch_bytes:
            raise RuntimeError("runtime did not apply the requested dispatch limit")
        if args.pdl:
            runtime.set_pdl(True)
        runtime.prepare((torch.bfloat16, torch.float32, torch.float16), padded_gather=True)
    comm = PolicyCommunicator(runtime, policy, device, world)
    capture_context = (lambda s: runtime.capture(stream=s)) if runtime else (lambda s: nullcontext())
    dtypes = [getattr(torch, d) for d in args.dtypes]

    with reporting_failure(runtime):
        total = world * (world + 1) // 2
        control = torch.tensor([rank + 1], device=device, dtype=torch.float32)
        dist.all_reduce(control)
        if control.item() != total:
            raise RuntimeError(f"NCCL control all-reduce returned {control.item()}, expected {total}")

        checks = []
        before = runtime.stats()["ops_posted"] if runtime else 0
        if not args.skip_correctness:
            checks = _correctness(comm, runtime, world, rank, device, dtypes, capture_context)
        numerical = _numerics(comm, args, world, rank, device) if args.numerics else []
        timings = _benchmark(comm, runtime, args, world, rank, device, cpu_group, capture_context, dtypes,
                             nvcounters) if args.benchmark else []
        stats = None
        if runtime:
            runtime.check_health()
            if not args.skip_correctness and world > 1 and runtime.stats()["ops_posted"] <= before:
                raise RuntimeError("no probe payload used the NVLink kernels")
            stats = {k: v for k, v in runtime.stats().items() if k not in ("status",)}
    environment = {k: v for k, v in sorted(os.environ.items()) if k.startswith(("SPARKNET_", "NCCL_"))}
    result = {"rank": rank, "world_size": world, "transport": args.transport, "pdl": bool(runtime and runtime.pdl),
              "policy": ({k: (dict(v) if isinstance(v, dict) else v) for k, v in policy.__dict__.items()}
                         if policy else None),
              "runtime": stats, "environment": environment, "passed": True, "checks": checks,
              "numerical_checks": numerical, "timings": timings, "gpu": torch.cuda.get_device_name(device)}
    text = json.dumps(result, default=str)
    if rank == 0:
        print(text, flush=True)
        if args.output:
            with open(args.output, "w") as handle:
                handle.write(text + "\n")
    if runtime:
        torch.cuda.synchronize()
        dist.barrier(group=cpu_group)
        runtime.close()
    dist.barrier(group=cpu_group)
    dist.destroy_process_group()
    return 0


def _exact_sum(parts):
    import torch

    acc = torch.zeros_like(parts[0], dtype=torch.float32)
    for p in parts:
        acc = acc + p.float()
    return acc.to(parts[0].dtype)


def _correctness(comm, runtime, world, rank, device, dtypes, capture_context):
    import torch

    checks = []
    for dtype in dtypes:
        lengths = {1, 17, 1024, 2 * 1024 * 1024 // dtype.itemsize}
        if runtime:
            for limit in (runtime.max_size, runtime.max_gather_bytes, runtime.dispatch_max_bytes):
                lengths.update(limit // dtype.itemsize + o for o in (-16 // dtype.itemsize, 0, 16 // dtype.itemsize))
        for length in sorted(lengths):
            if length * dtype.itemsize > 64 << 20:
                continue
            pattern = (torch.arange(length, device=device) % 7).to(dtype)
            local = pattern + rank + 1
            scattered = torch.cat([local + 8 * peer for peer in range(world)])

            def collect():
                return comm.all_reduce(local), comm.all_gather(local, dim=0), comm.reduce_scatter(scattered, dim=0)

            def verify(outputs, increment=0):
                ar, ag, rs = outputs
                torch.cuda.synchronize()
                ranks_local = [pattern + p + 1 + increment for p in range(world)]
                want_ar = _exact_sum(ranks_local)
                exact = comm.backend_for_all_reduce(local) != "nccl"
                if exact:
                    assert torch.equal(ar, want_ar), f"all-reduce {dtype} {length}"
                else:
                    torch.testing.assert_close(ar.float(), want_ar.float(), rtol=1e-2, atol=1.0)
                assert torch.equal(ag, torch.cat(ranks_local)), f"all-gather {dtype} {length}"
                chunks = [torch.cat([q + 8 * peer for peer in range(world)])[rank * length:(rank + 1) * length]
                          for q in ranks_local]
                torch.testing.assert_close(rs.float(), _exact_sum(chunks).float(), rtol=1e-2, atol=1.0)

            ledger0 = {k: list(v) for k, v in comm.ledger.items()}
            calls0 = dict(runtime.stats()["calls"]) if runtime is not None else {}
            verify(collect())
            if runtime is not None:
                check_runtime_counters(calls0, dict(runtime.stats()["calls"]), ledger0, comm.ledger,
                                       what=f"correctness {dtype} {length}")
            stream = torch.cuda.Stream(device=device)
            stream.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream), capture_context(stream):
                outputs = collect()
            for step in range(1, 5):
                local.add_(1)
                scattered.add_(1)
                graph.replay()
                verify(outputs, step)
            if runtime:
                runtime.check_health()
            checks.append({"dtype": str(dtype), "elements_per_rank": length, "eager": True, "graph_replays": 4,
                           "all_reduce_backend": comm.backend_for_all_reduce(local)})
            del graph, outputs, local, scattered, pattern
    return checks


def _numerics(comm, args, world, rank, device):
    import torch

    rows = []
    for dtype in (torch.bfloat16, torch.float32):
        base = torch.arange(64, dtype=torch.float32) % 8
        values = [(base + 1) * 16777216, (base + 1) / 16, -(base + 1) * 16777216, (base + 1) / 32]
        values = [values[i % 4] * (1 + i // 4) for i in range(world)]
        inputs = [v.to(dtype) for v in values]
        reference = _exact_sum([v.float() for v in inputs]).to(dtype)
        for length in args.lengths:
            local = inputs[rank].to(device).repeat((length + 63) // 64)[:length].contiguous()
            output = comm.all_reduce(local)
            torch.cuda.synchronize()
            observed = output[:64].cpu()
            rows.append({"dtype": str(dtype), "elements_per_rank": length,
                         "prefix_sha256": hashlib.sha256(observed.view(torch.uint8).numpy().tobytes()).hexdigest(),
                         "rank_order_fp32_prefix_sha256":
                             hashlib.sha256(reference.view(torch.uint8).numpy().tobytes()).hexdigest(),
                         "mismatched_reference_elements": int((observed != reference).sum())})
    return rows


def _benchmark(comm, runtime, args, world, rank, device, cpu_group, capture_context, dtypes, nvcounters):
    """Steady graph-replayed latency per (dtype, size, operation, arm), with two
    consistency checks per case: the runtime's call counters moved exactly as the
    routing implies (always), and, with ``--counter-samples``, the NVLink bytes that
    this job's GPUs sent during the timed replays cover what the NVLink route must send
    (checked for NVLink routes on several ranks; recorded for NCCL)."""
    import torch
    import torch.distributed as dist

    def arms_for(operation: str) -> list[str]:
        """The sweep's arms per operation (every algorithm the runtime has for it), else
        the policy's own choice."""
        if not args.sweep or runtime is None:
            return ["policy"]
        nvls = ["nvls"] if runtime.has_multicast else []
        if operation == "all_reduce":
            return ["oneshot", "twoshot"] + nvls + ["nccl"]
        if operation == "all_gather":
            return ["ll", "push"] + nvls + ["nccl"]
        return ["oneshot", "nccl"]
    calls_per_graph, replays_per_sample, samples_per_case = 16, 16, 5
    timings = []
    for dtype in dtypes:
        for length in args.lengths:
            nbytes = length * dtype.itemsize
            local = torch.full((length,), rank + 1, device=device, dtype=dtype)
            scattered = torch.cat([local + 8 * p for p in range(world)])
            for name in args.operations:
                for arm in arms_for(name):
                    op = _operation(comm, runtime, name, arm, local, scattered, nbytes)
                    if op is None:
                        continue
                    ledger0 = {k: list(v) for k, v in comm.ledger.items()}
                    calls0 = dict(runtime.stats()["calls"]) if runtime is not None else {}
                    op()
                    torch.cuda.synchronize()
                    stream = torch.cuda.Stream(device=device)
                    stream.wait_stream(torch.cuda.current_stream())
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=stream), capture_context(stream):
                        outputs = [op() for _ in range(calls_per_graph)]
                    route = comm.last_route
                    if runtime is not None:
                        check_runtime_counters(calls0, dict(runtime.stats()["calls"]), ledger0, comm.ledger,
                                               what=f"{name} [{arm}] {nbytes} B")
                    for _ in range(4):
                        graph.replay()
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu_group)
                    own_before = nvcounters.own_gpu_counters(device.index) if args.counter_samples else {}
                    samples = []
                    for _ in range(samples_per_case):
                        dist.barrier(group=cpu_group)
                        if runtime is not None:
                            runtime.barrier()
                        start = torch.cuda.Event(enable_timing=True)
                        end = torch.cuda.Event(enable_timing=True)
                        start.record()
                        for _ in range(replays_per_sample):
                            graph.replay()
                        end.record()
                        end.synchronize()
                        samples.append(start.elapsed_time(end) * 1000 / (calls_per_graph * replays_per_sample))
                    own_after = nvcounters.own_gpu_counters(device.index) if args.counter_samples else {}
                    tx = None
                    if "nvlink_tx_bytes" in own_before and "nvlink_tx_bytes" in own_after:
                        tx = own_after["nvlink_tx_bytes"] - own_before["nvlink_tx_bytes"]
                    gathered = [None] * world
                    dist.all_gather_object(gathered, (samples, tx), group=cpu_group)
                    slowest = [max(g[0][i] for g in gathered) for i in range(len(samples))]
                    row = {"dtype": str(dtype), "elements_per_rank": length, "operation": name, "arm": arm,
                           "backend": route.backend, "microseconds_per_call": slowest,
                           "median_us": statistics.median(slowest), "calls_per_graph": calls_per_graph,
                           "replays_per_sample": replays_per_sample}
                    if args.counter_samples:
                        timed_calls = calls_per_graph * replays_per_sample * samples_per_case
                        want = nvlink_bytes_expected(route, world) * timed_calls
                        seen = [g[1] for g in gathered]
                        row["nvlink_tx_bytes_per_rank"] = seen
                        row["nvlink_tx_bytes_expected_per_rank"] = want
                        row["nvlink_counter_source"] = own_after.get("source") or own_after.get("why")
                        if all(v is not None for v in seen) and route.nvlink and world > 1:
                            # NVLink counters count the payload plus protocol overhead;
                            # sending less than the payload means the route was not taken
                            short = [r for r, v in enumerate(seen) if v < 0.9 * want]
                            row["nvlink_counters_agree"] = not short
                            if short:
                                raise RuntimeError(f"{name} [{arm}] {nbytes} B: ranks {short} sent {seen} bytes "
                                                   f"over NVLink, the {route.backend} route needs {want} each")
                    if rank == 0:
                        print(json.dumps({"rank": rank, "timing": row}), flush=True)
                    timings.append(row)
                    del graph, outputs
            del local, scattered
    return timings


def _operation(comm, runtime, name, arm, local, scattered, nbytes):
    """A zero-argument callable for one (operation, arm), or None if the arm cannot carry
    it.  Every arm goes through the dispatcher, so its ledger sees every call."""
    if name == "all_reduce":
        if arm == "policy":
            return lambda: comm.all_reduce(local)
        if arm != "nccl":
            if runtime is None or nbytes > runtime.max_size:
                return None
            if arm == "oneshot" and nbytes > runtime._caps[0]:
                return None
            if arm == "nvls" and (not runtime.has_multicast or nbytes > runtime._mc[2]):
                return None
        return lambda: comm.all_reduce(local, algorithm=arm)
    if name == "all_gather" and arm in ("ll", "push", "nvls"):
        # the NVLink all-gather with its protocol forced: LL8 (flag in every 8-byte word),
        # the bulk push (flag per shard) or NVLS multicast stores
        if runtime is None or nbytes > runtime.max_gather_bytes or not runtime._gather_algorithm_fits(arm, nbytes):
            return None
        return lambda: comm.all_gather(local, dim=0, algorithm=arm)
    if name in ("all_gather", "reduce_scatter"):
        if arm not in ("policy", "oneshot", "nccl"):
            return None
        call = comm.all_gather if name == "all_gather" else comm.reduce_scatter
        tensor = local if name == "all_gather" else scattered
        return lambda: call(tensor, dim=0, force_nccl=(arm == "nccl"))
    return None


if __name__ == "__main__":
    sys.exit(main())
