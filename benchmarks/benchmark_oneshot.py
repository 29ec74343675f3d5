#!/usr/bin/env python3
"""NVLink collectives vs NCCL, eager and graph-replayed, interleaved arms.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/benchmark_oneshot.py --sizes 10240 61440 491520 2097152
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/benchmark_oneshot.py --fused-norm-tokens 1 8 32 128 256

``--arms nvlink-graph nvlink-pdl-graph nccl-graph`` adds the NVLink graph captured with
programmatic dependent launch (each call scheduled while the previous one runs).

With ``--fused-norm-tokens`` the arms are the decode epilogue instead: the fused NVLink
all-reduce + residual add + RMSNorm (hidden 8192, bf16, eps 1e-5) against NCCL's
all-reduce followed by this package's add + RMSNorm kernel (the same rounding points).

Method (after the reference's ``benchmarks/benchmark_oneshot.py``):

* correctness before and after timing: the NVLink all-reduce must equal the sequential
  rank-order fp32 sum bit for bit, and agree with NCCL within bf16 tolerance;
* arms are timed in interleaved blocks, with the arm order reversed on odd blocks, so
  drift (clocks, thermal) hits every arm alike;
* one sample = one arm for ``--calls`` back-to-back calls (a captured graph for the
  graph arms), device-timed with CUDA events; the cross-rank maximum of each sample
  is taken (every rank times the same sample), and the result is the median of those
  paired maxima, per call;
* the JSON receipt carries the git revision, GPU names, NCCL version and environment.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

ARMS = ("nvlink-graph", "nccl-graph", "nvlink-eager", "nccl-eager")
# also selectable: the NVLink graph captured with programmatic dependent launch
EXTRA_ARMS = ("nvlink-pdl-graph",)


def git_state() -> dict:
    try:
        rev = subprocess.run(["git", "rev-parse", "HEAD"], cwd=ROOT, capture_output=True, text=True).stdout.strip()
        dirty = bool(subprocess.run(["git", "status", "--porcelain"], cwd=ROOT, capture_output=True,
                                    text=True).stdout.strip())
        return {"revision": rev or None, "dirty": dirty}
    except OSError:
        return {"revision": None, "dirty": None}


def rank_order_sum(x: torch.Tensor, world: int) -> torch.Tensor:
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x)
    acc = torch.zeros_like(x, dtype=torch.float32)
    for p in parts:
        acc = acc + p.float()
    return acc.to(x.dtype)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--sizes", type=int, nargs="+", default=[10240, 61440, 491520, 2097152], help="bytes per rank")
    ap.add_argument("--blocks", type=int, default=6)
    ap.add_argument("--samples-per-block", type=int, default=3)
    ap.add_argument("--calls", type=int, default=64)
    ap.add_argument("--arms", nargs="+", default=list(ARMS), choices=ARMS + EXTRA_ARMS)
    ap.add_argument("--fused-norm-tokens", type=int, nargs="*", default=[],
                    help="time the fused all-reduce + residual + RMSNorm for these token counts instead")
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--output", default="")
    args = ap.parse_args()

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=120), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    cpu = dist.new_group(backend="gloo")
    from sparknet.oneshot import AllReduce

    rt = AllReduce.from_exchange_group(exchange_group=cpu, device=device, max_size=max(8 << 20, max(args.sizes)))
    rt.prepare((torch.bfloat16,))
    rows = []
    if args.fused_norm_tokens:
        rows = fused_norm_rows(args, rt, rank, world, device, cpu)
    for nbytes in ([] if args.fused_norm_tokens else args.sizes):
        gen = torch.Generator(device=device).manual_seed(nbytes + rank)
        x = torch.randn(nbytes // 2, generator=gen, device=device).to(torch.bfloat16)
        out = torch.empty_like(x)
        want = rank_order_sum(x, world)

        def check(tag):
            got = rt.all_reduce(x)
            ref = x.clone()
            dist.all_reduce(ref)
            torch.cuda.synchronize()
            if not torch.equal(got, want):
                raise RuntimeError(f"{tag}: NVLink all-reduce differs from the rank-order sum at {nbytes} B")
            if not torch.allclose(got.float(), ref.float(), rtol=2e-2, atol=2e-2 * world):
                raise RuntimeError(f"{tag}: NVLink and NCCL disagree at {nbytes} B")

        check("before")
        nccl_buf = x.clone()
        calls = {
            "nvlink-eager": lambda: rt.all_reduce(x, out=out),
            "nccl-eager": lambda: dist.all_reduce(nccl_buf),
        }
        graphs = {}
        stream = torch.cuda.Stream(device=device)
        for arm, fn in (("nvlink-graph", calls["nvlink-eager"]), ("nvlink-pdl-graph", calls["nvlink-eager"]),
                        ("nccl-graph", calls["nccl-eager"])):
            if arm not in args.arms:
                continue
            fn()
            torch.cuda.synchronize()
            stream.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            ctx = rt.capture(stream=stream) if arm.startswith("nvlink") else _Null()
            rt.set_pdl(arm == "nvlink-pdl-graph")  # the launch attribute is recorded in the graph
            with torch.cuda.graph(g, stream=stream), ctx:
                for _ in range(args.calls):
                    fn()
            rt.set_pdl(False)
            graphs[arm] = g
        samples = {arm: [] for arm in args.arms}
        for block in range(args.blocks):
            order = list(args.arms) if block % 2 == 0 else list(reversed(args.arms))
            for arm in order:
                for _ in range(args.samples_per_block):
                    dist.barrier(group=cpu)
                    rt.barrier()
                    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    st.record()
                    if arm in graphs:
                        graphs[arm].replay()
                    else:
                        for _ in range(args.calls):
                            calls[arm]()
                    en.record()
                    en.synchronize()
                    samples[arm].append(st.elapsed_time(en) * 1000.0 / args.calls)
        check("after")
        rt.check_health()
        gathered = [None] * world
        dist.all_gather_object(gathered, samples, group=cpu)
        row = {"bytes_per_rank": nbytes}
        for arm in args.arms:
            paired = [max(g[arm][i] for g in gathered) for i in range(len(samples[arm]))]
            row[arm] = {"median_us": statistics.median(paired), "samples": len(paired)}
        rows.append(row)
        del graphs
        torch.cuda.synchronize()
    receipt = {
        "benchmark": "benchmark_oneshot", "world_size": world, "rows": rows, "git": git_state(),
        "gpus": sorted({torch.cuda.get_device_name(device)}), "nccl": ".".join(map(str, torch.cuda.nccl.version())),
        "torch": torch.__version__, "time": time.time(),
        "environment": {k: v for k, v in sorted(os.environ.items()) if k.startswith(("SPARKNET_", "NCCL_"))},
    }
    if rank == 0:
        text = json.dumps(receipt)
        print(text, flush=True)
        if args.output:
            Path(args.output).write_text(text + "\n")
    dist.barrier(group=cpu)
    rt.close()
    dist.barrier(group=cpu)
    dist.destroy_process_group()
    return 0


def fused_norm_rows(args, rt, rank, world, device, cpu) -> list:
    """Interleaved arms for the decode epilogue: residual += all_reduce(x); y = RMSNorm(residual) * gamma."""
    from sparknet import _native

    C = _native.load()
    H, eps = args.hidden, 1e-5
    rows = []
    for tokens in args.fused_norm_tokens:
        gen = torch.Generator(device=device).manual_seed(1000 * tokens + rank)
        x = torch.randn(tokens, H, generator=gen, device=device).to(torch.bfloat16)
        res = torch.randn(tokens, H, generator=torch.Generator(device=device).manual_seed(tokens), device=device)
        res = res.to(torch.bfloat16)
        gamma = (1 + 0.02 * torch.randn(H, generator=torch.Generator(device=device).manual_seed(7),
                                        device=device)).to(torch.bfloat16)
        out_f, res_f = torch.empty_like(x), torch.empty_like(res)
        out_n, res_n, xn = torch.empty_like(x), torch.empty_like(res), x.clone()

        def fused():
            rt.all_reduce_residual_rmsnorm(x, res, gamma, eps, out=out_f, residual_out=res_f)

        def unfused():
            xn.copy_(x)
            dist.all_reduce(xn)
            C.add_rmsnorm(xn, res, res_n, gamma, out_n, eps)

        fused()
        unfused()
        torch.cuda.synchronize()
        if not torch.allclose(out_f.float(), out_n.float(), rtol=2e-2, atol=2e-2):
            raise RuntimeError(f"fused and unfused epilogues disagree at {tokens} tokens")
        arms = {"nvlink-fused": fused, "nccl-unfused": unfused}
        graphs = {}
        stream = torch.cuda.Stream(device=device)
        for name, fn in arms.items():
            stream.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            ctx = rt.capture(stream=stream) if name.startswith("nvlink") else _Null()
            with torch.cuda.graph(g, stream=stream), ctx:
                for _ in range(args.calls):
                    fn()
            graphs[name] = g
        samples = {name: [] for name in arms}
        for block in range(args.blocks):
            order = list(arms) if block % 2 == 0 else list(reversed(list(arms)))
            for name in order:
                for _ in range(args.samples_per_block):
                    dist.barrier(group=cpu)
                    rt.barrier()
                    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    st.record()
                    graphs[name].replay()
                    en.record()
                    en.synchronize()
                    samples[name].append(st.elapsed_time(en) * 1000.0 / args.calls)
        rt.check_health()
        gathered = [None] * world
        dist.all_gather_object(gathered, samples, group=cpu)
        row = {"tokens": tokens, "hidden": H}
        for name in arms:
            paired = [max(g[name][i] for g in gathered) for i in range(len(samples[name]))]
            row[name + "-graph"] = {"median_us": statistics.median(paired), "samples": len(paired)}
        rows.append(row)
        del graphs
        torch.cuda.synchronize()
    return rows


class _Null:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False


if __name__ == "__main__":
    sys.exit(main())
