"""One rank of the multi-process NVLink test (launched by torch.distributed.run).

Checks every collective of ``sparknet.oneshot.AllReduce`` against oracles built from
NCCL all-gathers of the inputs: all-reduce and reduce-scatter bit-exact against the
rank-order fp32 sum, all-gather/exchange/all_to_all_rows exact, the fused
all-reduce + RMSNorm bit-identical across ranks, graph replay, and (when the box has
NVLS) the multicast paths.  Prints one JSON line per rank.
"""

import hashlib
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def rank_order_sum(xs):
    acc = torch.zeros_like(xs[0], dtype=torch.float32)
    for x in xs:
        acc = acc + x.float()
    return acc.to(xs[0].dtype)


def gather_all(x, world):
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous())
    return parts


FAILURES = []


def expect(cond, msg):
    """Record a failed check without leaving the collective sequence early: every rank
    must reach the same teardown (a rank that exits while bound to a multicast object
    can disturb its peers)."""
    if not cond:
        FAILURES.append(msg)


def digest(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=60))
    from sparknet.oneshot import AllReduce

    nvls = os.environ.get("SPARKNET_NVLS") == "1"
    rt = AllReduce.from_exchange_group(exchange_group=cpu, device=device, max_size=8 << 20,
                                       max_gather_bytes=4 << 20, enable_multicast=nvls)
    rt.set_timeout_ms(5000)
    rt.prepare((torch.bfloat16, torch.float16, torch.float32), padded_gather=True)
    results = {"rank": rank, "world": world, "multicast": rt.has_multicast, "checks": 0}
    if nvls:
        print(f"rank {rank}: multicast available: {rt.has_multicast}", flush=True)
    algos = ["oneshot", "twoshot"] + (["nvls"] if rt.has_multicast else [])

    def check_same_everywhere(t, what):
        ds = [None] * world
        dist.all_gather_object(ds, digest(t), group=cpu)
        expect(len(set(ds)) == 1, f"{what}: ranks differ")

    gen = torch.Generator(device=device)
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        for nbytes in (16, 1024, 10 * 1024, 60 * 1024, 480 * 1024, 2 << 20, 8 << 20):
            numel = nbytes // torch.tensor([], dtype=dtype).element_size()
            gen.manual_seed(nbytes + rank)
            x = torch.randn(numel, generator=gen, device=device).to(dtype)
            want = rank_order_sum(gather_all(x, world))
            for algo in algos:
                if algo == "oneshot" and nbytes > rt._caps[0]:
                    continue
                out = rt.all_reduce(x, algorithm=algo)
                torch.cuda.synchronize()
                check_same_everywhere(out, f"all_reduce {algo} {dtype} {nbytes}")
                if algo != "nvls":
                    expect(torch.equal(out, want), f"all_reduce {algo} {dtype} {nbytes} != rank-order sum")
                else:
                    expect(torch.allclose(out.float(), want.float(), rtol=2e-2, atol=2e-2), f"nvls {dtype} {nbytes}")
                results["checks"] += 1
    # reduce-scatter
    for dtype in (torch.bfloat16, torch.float32):
        x = torch.randn(4 * world, 1024, generator=gen, device=device).to(dtype)
        out = rt.reduce_scatter(x)
        full = rank_order_sum(gather_all(x, world))
        expect(torch.equal(out, full[rank * 4:(rank + 1) * 4]), "reduce_scatter")
        results["checks"] += 1
    # all-gather: LL, push, padded, sliced
    for shape, dim in (((1, 64), 0), ((6, 5120), -1), ((96, 256), 0), ((600, 4096), 0), ((3, 7), -1),
                       ((4096, 1024), 0)):
        x = (torch.randn(shape, generator=gen, device=device) + rank).to(torch.bfloat16)
        sliced = x.numel() * 2 > rt.max_gather_bytes
        out = rt.all_gather(x, dim=dim, sliced=sliced)
        torch.cuda.synchronize()
        expect(torch.equal(out, torch.cat(gather_all(x, world), dim=dim)), f"all_gather {shape} {dim}")
        results["checks"] += 1
    # exchange and all_to_all_rows
    chunks = torch.randn(world, 16, 4096, generator=gen, device=device).to(torch.bfloat16)
    parts = torch.full_like(chunks, -7.0)
    rt.exchange(chunks, out=parts, copy_self=True)
    everyone = gather_all(chunks, world)
    for p in range(world):
        expect(torch.equal(parts[p], everyone[p][rank]), "exchange")
    rows = 7
    total = world * rows - 3
    inp = torch.randn(total, 1024, generator=gen, device=device).to(torch.bfloat16)
    out = rt.all_to_all_rows(inp, rows)
    allin = [torch.empty_like(inp) for _ in range(world)]
    dist.all_gather(allin, inp)
    mine = max(0, min(rows, total - rank * rows))
    for p in range(world):
        expect(torch.equal(out[p, :mine], allin[p][rank * rows: rank * rows + mine]), "all_to_all_rows")
    results["checks"] += 2
    # fused all-reduce + residual + RMSNorm
    hidden = 8192
    for tokens in (1, 8, 32, 128, 256):
        gen.manual_seed(tokens * 31 + rank)
        x = torch.randn(tokens, hidden, generator=gen, device=device).to(torch.bfloat16)
        g2 = torch.Generator(device=device).manual_seed(tokens)
        residual = torch.randn(tokens, hidden, generator=g2, device=device).to(torch.bfloat16)
        gamma = (1 + 0.02 * torch.randn(hidden, generator=g2, device=device)).to(torch.bfloat16)
        s = rank_order_sum(gather_all(x, world))
        want_res = (s.float() + residual.float()).to(torch.bfloat16)
        for algo in ("oneshot", "twoshot"):
            out, res = rt.all_reduce_residual_rmsnorm(x, residual, gamma, 1e-5, algorithm=algo)
            torch.cuda.synchronize()
            expect(torch.equal(res, want_res), f"fused residual {tokens} {algo}")
            check_same_everywhere(out, f"fused {tokens} {algo}")
            var = want_res.float().pow(2).mean(-1, keepdim=True)
            ref = (want_res.float() * torch.rsqrt(var + 1e-5) * gamma.float()).to(torch.bfloat16)
            expect(torch.allclose(out.float(), ref.float(), rtol=1e-2, atol=1e-2), f"fused norm {tokens} {algo}")
            results["checks"] += 1
    # graph replay, two sizes interleaved on one stream
    xs = [torch.randn(n, generator=gen, device=device).to(torch.bfloat16) for n in (5120, 245760)]
    outs = [torch.empty_like(x) for x in xs]
    stream = torch.cuda.Stream(device=device)
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream), rt.capture(stream=stream):
        for x, o in zip(xs, outs):
            rt.all_reduce(x, out=o)
    for step in range(4):
        for x in xs:
            x.add_(1)
        graph.replay()
        torch.cuda.synchronize()
        for x, o in zip(xs, outs):
            want = rank_order_sum(gather_all(x, world))
            if rt.algorithm_for(x.numel() * 2, x.dtype) == "nvls":  # switch order, not rank order
                expect(torch.allclose(o.float(), want.float(), rtol=2e-2, atol=2e-2), f"graph replay {step} (nvls)")
            else:
                expect(torch.equal(o, want), f"graph replay {step}")
    expect(rt.failure() is None, f"health: {rt.failure()}")
    results["checks"] += 1
    # ineligible inputs are refused on every rank alike (the caller then uses NCCL)
    expect(not rt.should_allreduce(torch.zeros(64, dtype=torch.int32, device=device)), "int32 eligible")
    expect(not rt.should_allreduce(torch.zeros(7, dtype=torch.bfloat16, device=device)), "14 bytes eligible")
    expect(not rt.should_allreduce(torch.zeros(64, 2, dtype=torch.bfloat16, device=device).t()), "strided eligible")
    big = (rt.dispatch_max_bytes // 2) + 8
    expect(not rt.should_allreduce(torch.zeros(big, dtype=torch.bfloat16, device=device)), "over dispatch eligible")
    results["checks"] += 1
    # eager calls alternating between two streams stay ordered (sequence numbers are shared)
    s1, s2 = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
    xs = [torch.randn(4096, generator=gen, device=device).to(torch.bfloat16) for _ in range(6)]
    torch.cuda.synchronize()
    outs = []
    for i, x in enumerate(xs):
        with torch.cuda.stream(s1 if i % 2 == 0 else s2):
            outs.append(rt.all_reduce(x))
    torch.cuda.synchronize()
    for x, o in zip(xs, outs):
        expect(torch.equal(o, rank_order_sum(gather_all(x, world))), "alternating streams")
    results["checks"] += 1
    # all-gather and all-reduce of two sizes mixed in one graph, replayed with new inputs
    ag_in = [torch.randn(n, generator=gen, device=device).to(torch.bfloat16) for n in (1024, 65536)]
    ar_in = [torch.randn(n, generator=gen, device=device).to(torch.bfloat16) for n in (2048, 131072)]
    ag_out = [torch.empty(world * x.numel(), dtype=x.dtype, device=device) for x in ag_in]
    ar_out = [torch.empty_like(x) for x in ar_in]
    stream.wait_stream(torch.cuda.current_stream())
    mixed = torch.cuda.CUDAGraph()
    with torch.cuda.graph(mixed, stream=stream), rt.capture(stream=stream):
        for a, ao, b, bo in zip(ag_in, ag_out, ar_in, ar_out):
            rt.all_gather(a, dim=0, out=ao)
            rt.all_reduce(b, out=bo)
    for step in range(3):
        for t in ag_in + ar_in:
            t.mul_(-1)
        mixed.replay()
        torch.cuda.synchronize()
        for a, ao in zip(ag_in, ag_out):
            expect(torch.equal(ao, torch.cat(gather_all(a, world))), f"mixed graph all_gather {step}")
        for b, bo in zip(ar_in, ar_out):
            want = rank_order_sum(gather_all(b, world))
            if rt.algorithm_for(b.numel() * 2, b.dtype) == "nvls":
                expect(torch.allclose(bo.float(), want.float(), rtol=2e-2, atol=2e-2), f"mixed graph nvls {step}")
            else:
                expect(torch.equal(bo, want), f"mixed graph all_reduce {step}")
    del mixed
    expect(rt.failure() is None, f"health after mixed graph: {rt.failure()}")
    results["checks"] += 1
    results["stats"] = {k: v for k, v in rt.stats().items()
                        if k in ("calls", "epoch", "transport", "bytes_pushed_per_peer", "nvls_bytes")}
    if rt.trace_path:
        from sparknet.oneshot import trace

        torch.cuda.synchronize()
        header, recs = trace.read(rt.trace_path)
        ph = trace.phases(header, recs)
        results["trace"] = {"collectives": ph["collectives"], "wait_us": ph.get("wait_us")}
        expect(ph["collectives"] > 10 and "wait_us" in ph, f"trace recorded {ph}")
    del graph
    results["failures"] = FAILURES
    torch.cuda.synchronize()
    dist.barrier(group=cpu)
    rt.close()
    dist.barrier(group=cpu)
    out_dir = os.environ.get("SPARKNET_TEST_OUT")
    if out_dir:  # one file per rank: ranks printing at once interleave their lines
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps(results))
    else:
        print(json.dumps(results), flush=True)
    dist.destroy_process_group()
    return 1 if FAILURES else 0


if __name__ == "__main__":
    sys.exit(main())
