"""The one-rank runtime (launched by torch.distributed.run with one process).

At world size 1 the all-reduce is the ``local`` algorithm: one copy kernel launched
with programmatic dependent launch.  Checks: every dtype and size returns the input's
exact bits (special values included); in place is a no-op; a misaligned input goes
through the alignment scratch; a CUDA graph of chained calls, each reading the
previous call's output, ends with the input's bits (each launch waits for its
predecessor); the protocol path still runs when forced; with programmatic dependent
launch on, a sequence of collectives (all-reduce, all-gather, fused norm,
reduce-scatter, barrier) gives the bits it gives without.  Writes one JSON file.
"""

import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

FAILURES = []


def expect(cond, msg):
    if not cond:
        FAILURES.append(msg)


def same_bits(a, b):
    return a.shape == b.shape and torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def main():
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    if dist.get_world_size() != 1:
        raise SystemExit("single_rank_worker runs with one process")
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=60))
    from sparknet.oneshot import AllReduce

    rt = AllReduce.from_exchange_group(exchange_group=cpu, device=device, max_size=8 << 20)
    rt.set_timeout_ms(2000)
    rt.prepare((torch.bfloat16, torch.float16, torch.float32))
    results = {"world": 1, "checks": 0}
    gen = torch.Generator(device=device).manual_seed(7)

    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        esize = torch.tensor([], dtype=dtype).element_size()
        for nbytes in (16, 10240, 61440, 491520, 2 << 20, 8 << 20):
            x = torch.randn(nbytes // esize, generator=gen, device=device).to(dtype)
            expect(rt.algorithm_for(nbytes, dtype) == "local", f"algorithm at {nbytes}")
            y = rt.all_reduce(x)
            torch.cuda.synchronize()
            expect(same_bits(y, x), f"{dtype} {nbytes}: copy differs")
            results["checks"] += 1

    # bit patterns a sum would canonicalise or a sentinel would collide with survive a copy
    raw = torch.arange(4096, device=device, dtype=torch.int32).to(torch.int16)
    raw[:8] = torch.tensor([-1, -32768, 0x7FC0, -64, 0x7F80, -128, 0, 1], dtype=torch.int16, device=device)
    special = raw.view(torch.bfloat16)
    expect(same_bits(rt.all_reduce(special), special), "special bit patterns")
    results["checks"] += 1

    # in place: no launch, the input already is the result
    x = torch.randn(4096, generator=gen, device=device).to(torch.bfloat16)
    keep = x.clone()
    expect(rt.all_reduce(x, out=x) is x and same_bits(x, keep), "in place")
    results["checks"] += 1

    # a misaligned view (8 bytes in) goes through the aligned scratch
    big = torch.randn(4096 + 4, generator=gen, device=device).to(torch.bfloat16)
    view = big[4:]
    expect(same_bits(rt.all_reduce(view), view), "misaligned input")
    results["checks"] += 1

    # graph: 64 chained calls, call k reading call k-1's output; every buffer but the
    # first is poisoned with NaN before each replay, so a launch that read before its
    # predecessor finished would carry NaN to the end
    n, chain = 1 << 20, 64
    bufs = [torch.randn(n, generator=gen, device=device).to(torch.bfloat16)] + \
        [torch.empty(n, device=device, dtype=torch.bfloat16) for _ in range(chain)]
    stream = torch.cuda.Stream(device=device)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for k in range(chain):
            rt.all_reduce(bufs[k], out=bufs[k + 1])
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream), rt.capture(stream=stream):
        for k in range(chain):
            rt.all_reduce(bufs[k], out=bufs[k + 1])
    for rep in range(5):
        for b in bufs[1:]:
            b.fill_(float("nan"))
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        expect(same_bits(bufs[-1], bufs[0]), f"graph chain replay {rep}")
        expect(all(same_bits(b, bufs[0]) for b in bufs[1:]), f"graph chain intermediates {rep}")
    results["checks"] += 1
    del graph

    stats = rt.stats()
    results["calls"] = stats["calls"]
    expect(stats["calls"]["local"] > 0 and stats["bytes_pushed_per_peer"] == 0, f"stats {stats['calls']}")

    # the protocol path, forced, still computes the same (one-rank sum = the input)
    x = torch.randn(8192, generator=gen, device=device).to(torch.float32)
    expect(same_bits(rt.all_reduce(x, algorithm="oneshot"), x), "forced one-shot at one rank")
    try:
        rt.all_reduce(x, algorithm="bogus")
        expect(False, "unknown algorithm accepted")
    except ValueError:
        pass
    results["checks"] += 1

    # programmatic dependent launch for the collective kernels: the same sequence of
    # collectives (protocol paths forced where one rank would copy) gives the same bits
    # with and without it, eagerly and replayed from a graph
    tokens, hidden = 16, 8192
    xa = torch.randn(tokens, hidden, generator=gen, device=device).to(torch.bfloat16)
    res = torch.randn(tokens, hidden, generator=gen, device=device).to(torch.bfloat16)
    gamma = torch.randn(hidden, generator=gen, device=device).to(torch.bfloat16)
    outs = {k: torch.empty(tokens, hidden, device=device, dtype=torch.bfloat16)
            for k in ("ar", "ag", "rs", "norm", "res")}

    def sequence():
        rt.all_reduce(xa, out=outs["ar"], algorithm="oneshot")
        rt.all_gather(outs["ar"], dim=0, out=outs["ag"])
        rt.all_reduce_residual_rmsnorm(outs["ag"], res, gamma, 1e-5, out=outs["norm"], residual_out=outs["res"])
        rt.reduce_scatter(outs["norm"], out=outs["rs"])
        rt.barrier()

    sequence()
    torch.cuda.synchronize()
    want = {k: v.clone() for k, v in outs.items()}
    rt.set_pdl(True)
    expect(rt.pdl and rt.stats()["pdl"], "set_pdl(True) took effect")
    for v in outs.values():
        v.fill_(float("nan"))
    sequence()
    torch.cuda.synchronize()
    expect(all(same_bits(outs[k], want[k]) for k in want), "PDL eager sequence")
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream), rt.capture(stream=stream):
        for _ in range(8):
            sequence()
    for rep in range(3):
        for v in outs.values():
            v.fill_(float("nan"))
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        expect(all(same_bits(outs[k], want[k]) for k in want), f"PDL graph replay {rep}")
    del graph
    rt.set_pdl(False)
    results["checks"] += 1

    torch.cuda.synchronize()
    expect(rt.failure() is None, f"health: {rt.failure()}")
    results["failures"] = FAILURES
    rt.close()
    out_dir = os.environ.get("SPARKNET_TEST_OUT")
    if out_dir:
        Path(out_dir, "rank0.json").write_text(json.dumps(results))
    else:
        print(json.dumps(results), flush=True)
    dist.destroy_process_group()
    return 1 if FAILURES else 0


if __name__ == "__main__":
    sys.exit(main())
