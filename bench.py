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
                   help="ours: launch the collectives with programmatic dependent launch (the default)")
    p.add_argument("--no-pdl", action="store_true",
                   help="ours: launch the collectives without programmatic dependent launch")
    p.add_argument("--batch", type=int, default=8, help="decode: sequences per step")
    p.add_argument("--attention", choices=("auto", "simt", "tcgen05"), default="auto",
                   help="decode: attention kernel (auto: tensor cores where their cluster merge fits one wave or from 32 sequence-head pairs)")
    p.add_argument("--layers", type=int, default=80, help="decode: decoder layers")
    p.add_argument("--fused-norm-tokens", type=int, nargs="*", default=[1, 8, 32, 128, 256],
                   help="ours: also time the fused all-reduce + residual + RMSNorm at these token counts "
                        "(hidden --hidden); none to skip")
    p.add_argument("--hidden", type=int, default=8192, help="fused norm: hidden size")
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


def rank_order_sum(x: torch.Tensor, world: int) -> torch.Tensor:
    """The all-reduce every rank must return: all ranks' inputs (gathered with NCCL)
    summed in rank order 0..W-1 in fp32 and rounded once to ``x.dtype``."""
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous())
    acc = parts[0].float()
    for p in parts[1:]:
        acc = acc + p.float()
    return acc.to(x.dtype)


def compare_exact(got: torch.Tensor, want: torch.Tensor, cpu_group, world: int) -> dict:
    """Bit equality with ``want`` on this rank, and the same digest on every rank."""
    equal = bool(torch.equal(got.view(torch.int16), want.view(torch.int16)))
    err = (got.float() - want.float()).abs().max().item()
    digest = hashlib.sha256(got.view(torch.int16).cpu().numpy().tobytes()).hexdigest()
    digests = [None] * world
    dist.all_gather_object(digests, (digest, equal), group=cpu_group)
    return {"bit_exact": all(e for _, e in digests), "rank_identical": len({d for d, _ in digests}) == 1,
            "max_abs_err_vs_rank_order_sum": err}


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
                 pdl: bool | None = None):
        self.impl, self.rank, self.world, self.device = impl, rank, world, device
        self.algorithm = algorithm
        self.launches_per_call = 1
        if impl == "ours":
            from sparknet import _native
            from sparknet.oneshot import AllReduce

            self.rt = AllReduce.from_exchange_group(exchange_group=cpu_group, device=device)
            if pdl is not None:
                self.rt.set_pdl(pdl)
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

    arm = Arm(args.impl, rank, world, device, cpu_group, args.algorithm,
              pdl=False if args.no_pdl else (True if args.pdl else None))
    flush = L2Flusher(device)
    sizes = [int(s) for s in args.sizes]
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    inputs = {s: torch.randn(s // 2, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
              for s in sizes}
    # correctness: every rank's output must equal, bit for bit, the fp32 sum of all
    # ranks' bf16 inputs taken in rank order and rounded once (the library's contract),
    # and be identical on every rank.  NVLS reduces inside the switch in no fixed
    # order, so a forced --algorithm nvls is held to a tolerance instead.
    exact_required = args.impl == "ours" and args.algorithm != "nvls"
    expected = {s: rank_order_sum(inputs[s], world) for s in sizes}
    checks = {}
    for s in sizes:
        got = arm.all_reduce(inputs[s])
        torch.cuda.synchronize()
        checks[s] = compare_exact(got, expected[s], cpu_group, world)
        if exact_required and not checks[s]["bit_exact"]:
            raise RuntimeError(f"all-reduce at {s} bytes is not the rank-order sum: {checks[s]}")
        if not checks[s]["rank_identical"] and args.impl == "ours":
            raise RuntimeError(f"all-reduce at {s} bytes differs across ranks")

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
    for s in sizes:  # the timed replays' last output is still the rank-order sum
        after = compare_exact(outs[s], expected[s], cpu_group, world)
        checks[s]["bit_exact_after_timing"] = after["bit_exact"]
        if exact_required and not after["bit_exact"]:
            raise RuntimeError(f"graph-replayed all-reduce at {s} bytes is not the rank-order sum: {after}")
    del graphs, outs  # graphs holding NCCL calls must go before the process group does
    torch.cuda.synchronize()

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(arm, args, sizes, rank, world, device, cpu_group)
    fused = None
    if args.impl == "ours" and args.fused_norm_tokens:
        try:
            fused = run_fused_norm(arm, args, rank, world, device, cpu_group)
        except RuntimeError as exc:  # a side measurement: recorded, the headline stands
            print(f"fused all-reduce + RMSNorm check failed: {exc}", file=sys.stderr, flush=True)
            fused = {"failed": str(exc)}

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
    if fused is not None:
        result["fused_allreduce_residual_rmsnorm"] = fused
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


def run_fused_norm(arm, args, rank, world, device, cpu_group):
    """The decode epilogue ``residual += all_reduce(x); out = RMSNorm(residual) * gamma``
    fused in one kernel, per token count: p50 per call (max over ranks) of a graph of 256
    calls, L2 flushed before each replay; beside it the unfused sequence of this library
    (one-shot/two-shot all-reduce, then the add + RMSNorm kernel).  Checks: the new
    residual equals the rank-order all-reduce plus the residual bit for bit, the output
    is identical on every rank, and it is within one bf16 rounding of an fp32 RMSNorm."""
    from sparknet import _native

    C = _native.load()
    L2Flusher = _local("timing").L2Flusher
    flush = L2Flusher(device)
    rt, H, eps = arm.rt, args.hidden, 1e-5
    rows = {}
    stream = torch.cuda.Stream(device=device)
    for tokens in args.fused_norm_tokens:
        gen = torch.Generator(device=device).manual_seed(5000 + 97 * tokens + rank)
        x = torch.randn(tokens, H, generator=gen, device=device).to(torch.bfloat16)
        shared = torch.Generator(device=device).manual_seed(77 + tokens)  # residual and gamma: same on all ranks
        res = torch.randn(tokens, H, generator=shared, device=device).to(torch.bfloat16)
        gamma = (1.0 + 0.02 * torch.randn(H, generator=shared, device=device)).to(torch.bfloat16)
        out, res_out = torch.empty_like(x), torch.empty_like(res)
        ar, out_u, res_u = torch.empty_like(x), torch.empty_like(x), torch.empty_like(res)
        rt.all_reduce_residual_rmsnorm(x, res, gamma, eps, out=out, residual_out=res_out,
                                       algorithm=rt._fused_norm_algorithm(tokens, x.numel() * x.element_size()))
        torch.cuda.synchronize()
        want_res = (rank_order_sum(x, world).float() + res.float()).to(torch.bfloat16)
        r32 = want_res.float()
        want_out = r32 * torch.rsqrt(r32.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()
        check = compare_exact(res_out, want_res, cpu_group, world)
        same_out = compare_exact(out, out, cpu_group, world)["rank_identical"]
        rel = ((out.float() - want_out).abs() / want_out.abs().clamp_min(1e-3)).max().item()
        rel = max(gather_floats([rel], cpu_group), key=lambda v: v[0])[0]  # the same verdict on every rank
        check.update({"out_rank_identical": same_out, "out_max_rel_err_vs_fp32": rel})
        if not (check["bit_exact"] and same_out and rel <= 2.0 ** -7):
            raise RuntimeError(f"fused all-reduce + RMSNorm at {tokens} tokens failed its checks: {check}")

        algo = rt._fused_norm_algorithm(tokens, x.numel() * x.element_size())

        def fused():  # the single kernel, at every token count (the API switches to the pair above a threshold)
            rt.all_reduce_residual_rmsnorm(x, res, gamma, eps, out=out, residual_out=res_out, algorithm=algo)

        def unfused():
            rt.all_reduce(x, out=ar)
            C.add_rmsnorm(ar, res, res_u, gamma, out_u, eps)

        graphs = {}
        for name, fn in (("fused", fused), ("unfused", unfused)):
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream), rt.capture(stream=stream):
                for _ in range(CALLS_PER_GRAPH):
                    fn()
            graphs[name] = g
        samples = {name: [] for name in graphs}
        cur = torch.cuda.current_stream()
        for step in range(args.warmup + args.steps):
            for name, g in graphs.items():
                flush()
                rt.barrier()
                st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                st.record(cur)
                g.replay()
                en.record(cur)
                if step >= args.warmup:
                    samples[name].append((st, en))
        torch.cuda.synchronize()
        rt.check_health()
        if not compare_exact(res_out, want_res, cpu_group, world)["bit_exact"]:
            raise RuntimeError(f"graph-replayed fused norm at {tokens} tokens changed its residual output")
        flat = [st.elapsed_time(en) for name in graphs for (st, en) in samples[name]]
        gathered = gather_floats(flat, cpu_group)
        row = {"check": check}
        for ni, name in enumerate(graphs):
            per = [max(g[ni * args.steps + k] for g in gathered) for k in range(args.steps)]
            row[f"{name}_p50_us"] = round(statistics.median(per) * 1000.0 / CALLS_PER_GRAPH, 3)
        row["algorithm"] = algo
        row["api_runs"] = "fused kernel" if tokens <= rt.fused_norm_max_tokens() else "all-reduce + add/RMSNorm kernel"
        rows[str(tokens)] = row
        del graphs
        torch.cuda.synchronize()
    return {"hidden": H, "dtype": "bf16", "calls_per_graph": CALLS_PER_GRAPH,
            "unfused": "this library's all_reduce then its add+RMSNorm kernel", "per_tokens": rows}


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
