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
from datetime import timedelta


def _policy_from_environment():
    from sparknet.policy import NVLINK_POLICY, CollectivePolicy

    env = dict(os.environ)
    if env.get("SPARKNET_ALLREDUCE_CAPACITY_BYTES") and env.get("SPARKNET_ALLGATHER_MAX_BYTES"):
        return CollectivePolicy.from_environment(env)
    return NVLINK_POLICY


class PolicyCommunicator:
    """The explicit policy over torch.distributed (NCCL) and the NVLink runtime."""

    def __init__(self, runtime, policy, device, world_size):
        import torch
        import torch.distributed as dist

        self._torch, self._dist = torch, dist
        self.runtime, self.policy, self.device, self.world_size = runtime, policy, device, world_size

    @staticmethod
    def _dtype_name(t) -> str:
        return str(t.dtype).replace("torch.", "")

    def backend_for_all_reduce(self, tensor) -> str:
        if self.runtime is None:
            return "nccl"
        nbytes = tensor.numel() * tensor.element_size()
        return self.policy.all_reduce_backend(nbytes, self._dtype_name(tensor), contiguous=tensor.is_contiguous(),
                                              world=self.world_size)

    def all_reduce(self, tensor, *, algorithm: str | None = None):
        backend = algorithm or self.backend_for_all_reduce(tensor)
        if backend != "nccl":
            if algorithm is None and not self.runtime.should_allreduce(tensor):
                raise RuntimeError("policy and runtime eligibility disagree for all-reduce")
            return self.runtime.all_reduce(tensor, algorithm=backend)
        out = tensor.clone()
        self._dist.all_reduce(out)
        return out

    def all_gather(self, tensor, dim=0, *, force_nccl: bool = False):
        nbytes = tensor.numel() * tensor.element_size()
        if (not force_nccl and self.runtime is not None
                and self.policy.all_gather_backend(nbytes, self._dtype_name(tensor), dim=dim, ndim=tensor.dim(),
                                                   contiguous=tensor.is_contiguous()) == "oneshot"):
            if not self.runtime.should_all_gather(tensor, dim):
                raise RuntimeError("policy and runtime eligibility disagree for all-gather")
            return self.runtime.all_gather(tensor, dim=dim)
        parts = [self._torch.empty_like(tensor) for _ in range(self.world_size)]
        self._dist.all_gather(parts, tensor.contiguous())
        return self._torch.cat(parts, dim=dim)

    def reduce_scatter(self, tensor, dim=0, *, force_nccl: bool = False):
        if dim != 0:
            raise ValueError("reduce-scatter is tested along dim 0")
        nbytes = tensor.numel() * tensor.element_size()
        if (not force_nccl and self.runtime is not None
                and self.policy.reduce_scatter_backend(nbytes, self.policy.all_reduce_capacity_bytes) == "oneshot"
                and self.runtime.should_reduce_scatter(tensor)):
            return self.runtime.reduce_scatter(tensor)
        out = self._torch.empty((tensor.shape[0] // self.world_size,) + tuple(tensor.shape[1:]), dtype=tensor.dtype,
                                device=tensor.device)
        self._dist.reduce_scatter_tensor(out, tensor.contiguous())
        return out


@contextmanager
def reporting_failure(runtime):
    """Re-raise whatever follows a failed collective with the runtime's failure report."""
    try:
        yield
    except Exception as error:
        report = runtime.failure() if runtime is not None else None
        if report is not None:
            raise RuntimeError(report) from error
        raise


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

            verify(collect())
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
    import torch
    import torch.distributed as dist

    arms = ["policy"]
    if args.sweep and runtime is not None:
        arms = ["oneshot", "twoshot"] + (["nvls"] if runtime.has_multicast else []) + ["nccl"]
    timings = []
    use_counters = args.counter_samples
    for dtype in dtypes:
        for length in args.lengths:
            nbytes = length * dtype.itemsize
            local = torch.full((length,), rank + 1, device=device, dtype=dtype)
            scattered = torch.cat([local + 8 * p for p in range(world)])
            for name in args.operations:
                for arm in arms:
                    op = _operation(comm, runtime, name, arm, local, scattered, nbytes)
                    if op is None:
                        continue
                    op()
                    torch.cuda.synchronize()
                    stream = torch.cuda.Stream(device=device)
                    stream.wait_stream(torch.cuda.current_stream())
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=stream), capture_context(stream):
                        outputs = [op() for _ in range(16)]
                    for _ in range(4):
                        graph.replay()
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu_group)
                    counters_before = nvcounters.nvlink_counters() if use_counters and rank == 0 else None
                    samples = []
                    for _ in range(5):
                        dist.barrier(group=cpu_group)
                        if runtime is not None:
                            runtime.barrier()
                        start = torch.cuda.Event(enable_timing=True)
                        end = torch.cuda.Event(enable_timing=True)
                        start.record()
                        for _ in range(16):
                            graph.replay()
                        end.record()
                        end.synchronize()
                        samples.append(start.elapsed_time(end) * 1000 / 256)
                    gathered = [None] * world
                    dist.all_gather_object(gathered, samples, group=cpu_group)
                    slowest = [max(g[i] for g in gathered) for i in range(len(samples))]
                    row = {"dtype": str(dtype), "elements_per_rank": length, "operation": name, "arm": arm,
                           "microseconds_per_call": slowest, "median_us": statistics.median(slowest),
                           "calls_per_graph": 16, "replays_per_sample": 16}
                    if counters_before is not None:
                        after = nvcounters.nvlink_counters()
                        row["nvlink_deltas"] = nvcounters.deltas(counters_before, after)
                        row["nvlink_error_deltas"] = nvcounters.error_deltas(counters_before, after)
                    if rank == 0:
                        print(json.dumps({"rank": rank, "timing": row}), flush=True)
                    timings.append(row)
                    del graph, outputs
            del local, scattered
    return timings


def _operation(comm, runtime, name, arm, local, scattered, nbytes):
    """A zero-argument callable for one (operation, arm), or None if the arm cannot carry it."""
    if name == "all_reduce":
        if arm == "policy":
            return lambda: comm.all_reduce(local)
        if arm == "nccl":
            return lambda: comm.all_reduce(local, algorithm="nccl")
        if runtime is None or nbytes > runtime.max_size:
            return None
        if arm == "oneshot" and nbytes > runtime._caps[0]:
            return None
        if arm == "nvls" and (not runtime.has_multicast or nbytes > runtime._mc[2]):
            return None
        return lambda: runtime.all_reduce(local, algorithm=arm)
    if name == "all_gather":
        if arm in ("policy", "oneshot"):
            return lambda: comm.all_gather(local, dim=0)
        if arm == "nccl":
            return lambda: comm.all_gather(local, dim=0, force_nccl=True)
        return None
    if name == "reduce_scatter":
        if arm in ("policy", "oneshot"):
            return lambda: comm.reduce_scatter(scattered, dim=0)
        if arm == "nccl":
            return lambda: comm.reduce_scatter(scattered, dim=0, force_nccl=True)
        return None
    return None


if __name__ == "__main__":
    sys.exit(main())
