#!/usr/bin/env python3
"""Headline benchmark: bf16 all-reduce p50 latency (max over ranks) at 10 KiB-2 MiB.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--workload allreduce|decode]

For N > 1 launch one rank per GPU with ``torch.distributed.run`` (``--master-addr
127.0.0.1``).  Method (the reference's probe method, ``sparknet/probe/collectives.py``
of the reference): per-rank bf16 inputs drawn N(0,1) from a per-rank seed, one CUDA
graph of 256 all-reduce calls per size, timed with CUDA events on the launching
stream; one step replays the graph of every size once.  L2 is flushed (a 256 MiB
write) before every replay, outside the timed events.  Ranks are aligned by one
untimed collective before each replay.  Per (step, size) the slowest rank's time is
kept; the p50 over steps divided by 256 is the per-call latency.  ``value`` is the
geometric mean of the four headline sizes' p50 (lower is better).

``--impl reference`` runs the unmodified reference from ``baseline/_ref`` through its
own public NCCL-only arm (``sparknet.probe.collectives.PolicyCommunicator`` with no
one-shot runtime: ``clone`` + ``torch.distributed.all_reduce`` on NCCL), with NCCL's
stock environment (NVLink/NVLS enabled).  ``--reference-env profile`` applies the
reference's ``direct-nccl-only`` profile environment instead (NCCL forced onto IB).

``e2e`` repeats the measurement through the public API end to end: every call copies
its input from pinned host memory, all-reduces eagerly and copies the result back.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
HEADLINE_SIZES = (10 * 1024, 60 * 1024, 480 * 1024, 2 * 1024 * 1024)
CALLS_PER_GRAPH = 256
METRIC = "bf16 all-reduce p50 µs (max over ranks) @10K–2MiB, 2/4/8 B200; TP8 decode tok/s"
# The reference's published one-shot latencies (GB10 + RoCE; its README.md:29-42),
# geometric mean of the four headline sizes, by world size; the bar on B200 is the
# NCCL arm measured alongside.
PUBLISHED_GEOMEAN_US = {2: (10.9 * 17.0 * 43.1 * 137.1) ** 0.25, 4: (16.9 * 28.0 * 94.0 * 307.7) ** 0.25}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("allreduce", "decode"), default="allreduce")
    p.add_argument("--sizes", type=int, nargs="*", default=list(HEADLINE_SIZES), help="bytes per rank")
    p.add_argument("--reference-env", choices=("stock", "profile"), default="stock")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--algorithm", default=None, help="force oneshot|twoshot|nvls (ours)")
    p.add_argument("--pdl", action="store_true",
                   help="ours: launch the collectives with programmatic dependent launch")
    p.add_argument("--batch", type=int, default=8, help="decode: sequences per step")
    p.add_argument("--fuse-gemm-ar", action="store_true",
                   help="decode: the O / down GEMM epilogues push into the all-reduce (NVLink arm)")
    p.add_argument("--prefetch", action="store_true",
                   help="decode: prefetch the next GEMM's weights into L2 during attention and the all-reduces")
    p.add_argument("--attention", choices=("split", "cluster"), default="split",
                   help="decode: span merge through a workspace (split) or a thread-block cluster")
    p.add_argument("--layers", type=int, default=80, help="decode: decoder layers")
    p.add_argument("--json-out", default="")
    return p.parse_args(argv)


ARGS = parse_args()

if ARGS.impl == "reference":
    # The reference and this repository share the import name ``sparknet``: put the
    # installed reference first and drop this checkout from the path.
    ref = ROOT / "baseline" / "_ref"
    sys.path[:] = [str(ref)] + [p for p in sys.path if p not in ("", str(ROOT), os.getcwd())]
    if ARGS.reference_env == "profile":
        from sparknet.nccl.profiles import environment as _ref_env  # the reference's

        for k, v in _ref_env("direct-nccl-only").items():
            if k.startswith("NCCL_"):
                os.environ[k] = v

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def _local(name: str):
    """This checkout's ``sparknet/utils/<name>.py``, loaded by path: under
    ``--impl reference`` the name ``sparknet`` belongs to the reference."""
    import importlib.util

    mod_name = f"_bench_{name}"
    if mod_name in sys.modules:
        return sys.modules[mod_name]
    spec = importlib.util.spec_from_file_location(mod_name, ROOT / "sparknet" / "utils" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[mod_name] = mod
    spec.loader.exec_module(mod)
    return mod


def _reference_available() -> str | None:
    ref = ROOT / "baseline" / "_ref" / "sparknet"
    if not ref.exists():
        return "baseline/_ref is not installed (pip install --target baseline/_ref of the reference failed)"
    return None


def setup(n_gpus: int):
    if "RANK" not in os.environ:
        os.environ.update({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0", "MASTER_ADDR": "127.0.0.1"})
        if "MASTER_PORT" not in os.environ:
            import socket

            with socket.socket() as s:
                s.bind(("127.0.0.1", 0))
                os.environ["MASTER_PORT"] = str(s.getsockname()[1])
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    from datetime import timedelta

    dist.init_process_group(backend="cpu:gloo,cuda:nccl", timeout=timedelta(seconds=120), device_id=device)
    cpu_group = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    return rank, world, device, cpu_group


def gather_floats(values: list[float], cpu_group) -> list[list[float]]:
    out: list = [None] * dist.get_world_size()
    dist.all_gather_object(out, values, group=cpu_group)
    return out


def clocks_gpus(world: int) -> list[int]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if all(v.strip().isdigit() for v in ids):
            return [int(v) for v in ids[:world]]
    return list(range(world))


class Arm:
    """One implementation: how to all-reduce, align ranks and capture."""

    def __init__(self, impl: str, rank: int, world: int, device, cpu_group, algorithm: str | None,
                 pdl: bool = False):
        self.impl, self.rank, self.world, self.device = impl, rank, world, device
        self.algorithm = algorithm
        self.launches_per_call = 1
        if impl == "ours":
            from sparknet import _native
            from sparknet.oneshot import AllReduce

            self.rt = AllReduce.from_exchange_group(exchange_group=cpu_group, device=device)
            if pdl:
                self.rt.set_pdl(True)
            self.rt.prepare((torch.bfloat16,))
            self.native_path = _native.loaded_path()
            self.align_buf = torch.zeros(8, dtype=torch.bfloat16, device=device)
        else:
            from sparknet.probe.collectives import PolicyCommunicator  # the reference's public arm

            self.comm = PolicyCommunicator(None, None, device, world)
            self.native_path = None
            self.align_buf = torch.zeros(8, dtype=torch.float32, device=device)

    def all_reduce(self, x, out=None):
        if self.impl == "ours":
            return self.rt.all_reduce(x, out=out, algorithm=self.algorithm)
        return self.comm.all_reduce(x)

    def align(self):
        """One untimed collective so every rank starts the timed work together."""
        if self.impl == "ours":
            self.rt.barrier()
        else:
            dist.all_reduce(self.align_buf)

    def capture_ctx(self, stream):
        import contextlib

        return self.rt.capture(stream=stream) if self.impl == "ours" else contextlib.nullcontext()


def run_allreduce(args, rank, world, device, cpu_group):
    ClockSampler = _local("clocks").ClockSampler
    L2Flusher, geomean = _local("timing").L2Flusher, _local("timing").geomean

    arm = Arm(args.impl, rank, world, device, cpu_group, args.algorithm, pdl=args.pdl)
    flush = L2Flusher(device)
    sizes = [int(s) for s in args.sizes]
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    inputs = {s: torch.randn(s // 2, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
              for s in sizes}
    # correctness against NCCL on the same inputs (tolerance: NCCL's order differs), and
    # identical bits on every rank
    checks = {}
    for s in sizes:
        got = arm.all_reduce(inputs[s])
        ref = inputs[s].float().clone()
        dist.all_reduce(ref)
        torch.cuda.synchronize()
        err = (got.float() - ref).abs().max().item()
        digest = hashlib.sha256(got.view(torch.int16).cpu().numpy().tobytes()).hexdigest()
        digests = [None] * world
        dist.all_gather_object(digests, digest, group=cpu_group)
        checks[s] = {"max_abs_err_vs_fp32": err, "rank_identical": len(set(digests)) == 1}
        if err > 1.0 + 0.25 * world:  # gross errors only: NCCL's bf16 order differs
            raise RuntimeError(f"all-reduce mismatch at {s} bytes: max error {err}")

    stream = torch.cuda.Stream(device=device)
    graphs, outs = {}, {}
    for s in sizes:
        out = torch.empty_like(inputs[s])
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(3):  # warm the call path on the capture stream
                r = arm.all_reduce(inputs[s], out=out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream), arm.capture_ctx(stream):
            for _ in range(CALLS_PER_GRAPH):
                r = arm.all_reduce(inputs[s], out=out)
        graphs[s], outs[s] = g, r
    torch.cuda.synchronize()

    def one_step(record: bool):
        times = []
        cur = torch.cuda.current_stream()
        for s in sizes:
            flush()
            arm.align()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(cur)
            graphs[s].replay()
            end.record(cur)
            times.append((start, end))
        return times

    # clocks: the sampler starts before the warm-up (nvidia-smi takes a moment to begin);
    # only samples stamped in the timed window (or nearest to a short one) count
    sampler = ClockSampler(clocks_gpus(world), interval_ms=20).start() if rank == 0 else None
    if sampler:
        time.sleep(0.5)  # nvidia-smi takes a moment to begin sampling
    for _ in range(args.warmup):
        one_step(False)
    torch.cuda.synchronize()
    dist.barrier(group=cpu_group)
    torch.cuda.synchronize()
    dist.barrier(group=cpu_group)
    if sampler:
        sampler.mark_start()
    t0 = time.perf_counter()
    recorded = [one_step(True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    dist.barrier(group=cpu_group)
    wall = time.perf_counter() - t0
    if sampler:
        sampler.mark_end()
    clocks = sampler.stop() if sampler else None
    per_rank = [[st.elapsed_time(en) for (st, en) in step] for step in recorded]  # ms [step][size]
    gathered = gather_floats([v for step in per_rank for v in step], cpu_group)
    n = len(sizes)
    p50_us, step_ms = {}, []
    for si, s in enumerate(sizes):
        samples = [max(g[k * n + si] for g in gathered) for k in range(args.steps)]
        p50_us[s] = statistics.median(samples) * 1000.0 / CALLS_PER_GRAPH
    for k in range(args.steps):
        step_ms.append(sum(max(g[k * n + si] for g in gathered) for si in range(n)))
    if args.impl == "ours":
        arm.rt.check_health()
    del graphs, outs  # graphs holding NCCL calls must go before the process group does
    torch.cuda.synchronize()

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(arm, args, sizes, rank, world, device, cpu_group)

    headline = [p50_us[s] for s in sizes if s in HEADLINE_SIZES] or list(p50_us.values())
    value = geomean(headline)
    result = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "us (geometric mean of per-size p50 per call)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(statistics.median(step_ms), 4),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": (round(value / PUBLISHED_GEOMEAN_US[world], 4) if world in PUBLISHED_GEOMEAN_US else None),
        "dtype": "bf16",
        "data": "synthetic N(0,1) per-rank seeded inputs",
        "config": {
            "model": "collective microbenchmark (no model)",
            "sizes_bytes_per_rank": sizes,
            "calls_per_graph": CALLS_PER_GRAPH,
            "global_batch": None,
            "seq_len": None,
            "parallelism": f"tp{world}",
            "l2": "flushed (256 MiB write) before every timed graph replay",
            "timing": "CUDA events per graph replay, max over ranks per step, p50 over steps",
        },
        "p50_us_per_size": {str(s): round(v, 3) for s, v in p50_us.items()},
        "checks": {str(s): v for s, v in checks.items()},
        "gpu_launches": args.steps * len(sizes) * CALLS_PER_GRAPH * arm.launches_per_call,
        "wall_s_timed": round(wall, 3),
        "clocks": clocks,
        "e2e": e2e,
    }
    if args.impl == "ours":
        result["algorithms"] = {str(s): (args.algorithm or arm.rt.algorithm_for(s, torch.bfloat16)) for s in sizes}
        result["native_extension"] = arm.native_path
        result["pdl"] = bool(arm.rt.pdl)
    else:
        result["impl"] = "reference"
        result["reference_arm"] = ("PolicyCommunicator(runtime=None): clone + torch.distributed.all_reduce (NCCL), "
                                   f"env={args.reference_env}")
        result["gpu_launches_note"] = "reference arm: NCCL library kernels, not this repository's"
    return result


def run_e2e(arm, args, sizes, rank, world, device, cpu_group):
    """Per call: pinned H2D of the input, eager all-reduce via the public API, D2H of the result."""
    geomean = _local("timing").geomean

    host_in = {s: torch.randn(s // 2, dtype=torch.float32).to(torch.bfloat16).pin_memory() for s in sizes}
    host_out = {s: torch.empty(s // 2, dtype=torch.bfloat16).pin_memory() for s in sizes}
    dev_in = {s: torch.empty(s // 2, dtype=torch.bfloat16, device=device) for s in sizes}
    dev_out = {s: torch.empty(s // 2, dtype=torch.bfloat16, device=device) for s in sizes}
    reps = 32
    cur = torch.cuda.current_stream()

    def once(s):
        dev_in[s].copy_(host_in[s], non_blocking=True)
        if arm.impl == "ours":
            arm.all_reduce(dev_in[s], out=dev_out[s])
            res = dev_out[s]
        else:
            res = arm.all_reduce(dev_in[s])
        host_out[s].copy_(res, non_blocking=True)

    for s in sizes:
        for _ in range(3):
            once(s)
    torch.cuda.synchronize()
    samples = {s: [] for s in sizes}
    for _ in range(max(3, args.steps)):
        for s in sizes:
            arm.align()
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record(cur)
            for _ in range(reps):
                once(s)
            en.record(cur)
            en.synchronize()  # the host reads the result
            samples[s].append(st.elapsed_time(en) * 1000.0 / reps)
    flat = [v for s in sizes for v in samples[s]]
    gathered = gather_floats(flat, cpu_group)
    k = len(samples[sizes[0]])
    p50 = {}
    for si, s in enumerate(sizes):
        per = [max(g[si * k + i] for g in gathered) for i in range(k)]
        p50[s] = statistics.median(per)
    headline = [p50[s] for s in sizes if s in HEADLINE_SIZES] or list(p50.values())
    return {
        "value": round(geomean(headline), 3),
        "unit": "us per call (geometric mean of per-size p50), pinned H2D + all_reduce + D2H",
        "p50_us_per_size": {str(s): round(v, 3) for s, v in p50.items()},
        "h2d_bytes_per_step": int(sum(sizes)),
        "d2h_bytes_per_step": int(sum(sizes)),
        "api": "sparknet.oneshot.AllReduce.all_reduce" if arm.impl == "ours"
        else "sparknet.probe.collectives.PolicyCommunicator.all_reduce (reference)",
    }


def main():
    args = ARGS
    if args.impl == "reference":
        why = _reference_available()
        if why:
            print(json.dumps({"impl": "reference", "unavailable": why}))
            return 0
    if args.workload == "decode":
        from sparknet.models.bench_decode import run_decode_bench  # noqa: WPS433

        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference has no model code; its NCCL-only arm is measured by the collective "
                              "workload"}))
            return 0
        rank, world, device, cpu_group = setup(args.gpus)
        result = run_decode_bench(args, rank, world, device, cpu_group)
    else:
        rank, world, device, cpu_group = setup(args.gpus)
        result = run_allreduce(args, rank, world, device, cpu_group)
    if rank == 0:
        line = json.dumps(result)
        print(line, flush=True)
        if args.json_out:
            Path(args.json_out).write_text(line + "\n")
    dist.barrier(group=cpu_group)
    torch.cuda.synchronize()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
