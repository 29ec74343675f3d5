#!/usr/bin/env python3
"""Fail-stop qualification: a rank that stops taking part must stop its peers,
within bounds, naming it, without faulting or hanging any GPU.

One child process per rank (one GPU each).  After healthy warm-up collectives the
victim rank skips one collective on the host (it stays alive and launches nothing);
every other rank's kernel waits, gives up after the runtime timeout, records the
victim in pinned memory and returns.  Each survivor must report the victim within
``0.9 x timeout`` to ``3 x timeout + 2 s`` (the reference's bounds,
``sparknet/probe/failstop.py:116-130``).  Then every rank re-arms collectively
(``reset``) and a healthy collective must give exact results: the context survived.
Graph mode does the same with a captured all-reduce that the victim does not replay.

Unlike the reference this never traps the GPU: waits end in a status word.  NVLS is
off (``NCCL_NVLS_ENABLE=0``, no multicast) so no rank is bound to a multicast object.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

SETUP_TIMEOUT_S = 120


def problems(result: dict, timeout_ms: int) -> list[str]:
    """Bounds on one survivor's report."""
    errors = []
    low, high = 0.9 * timeout_ms / 1000, 3 * timeout_ms / 1000 + 2.0
    for mode in ("eager", "graph"):
        r = result.get(mode)
        if r is None:
            continue
        if r.get("victim"):
            continue
        if not r.get("detected"):
            errors.append(f"{mode}: rank {result['rank']} did not detect the missing peer")
            continue
        if not low <= r["seconds"] <= high:
            errors.append(f"{mode}: rank {result['rank']} stopped after {r['seconds']:.2f} s, outside "
                          f"[{low:.2f}, {high:.2f}]")
        if f"waiting for rank {result['victim']}" not in r.get("report", ""):
            errors.append(f"{mode}: rank {result['rank']}'s report does not name rank {result['victim']}: "
                          f"{r.get('report')}")
        if not r.get("recovered"):
            errors.append(f"{mode}: rank {result['rank']} did not recover after reset")
    return errors


def _child(rank: int, world: int, port: int, timeout_ms: int, victim: int, queue) -> None:
    os.environ.update({"NCCL_NVLS_ENABLE": "0", "SPARKNET_NVLS": "0", "MASTER_ADDR": "127.0.0.1",
                       "MASTER_PORT": str(port), "RANK": str(rank), "WORLD_SIZE": str(world)})
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    out = {"rank": rank, "victim": victim}
    try:
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=SETUP_TIMEOUT_S))
        from sparknet.oneshot import AllReduce

        rt = AllReduce.from_exchange_group(exchange_group=dist.group.WORLD, device=device, max_size=1 << 20,
                                           max_gather_bytes=1 << 20, enable_multicast=False)
        rt.set_timeout_ms(timeout_ms)
        x = torch.full((8192,), float(rank + 1), device=device, dtype=torch.bfloat16)
        want = float(world * (world + 1) // 2)
        for _ in range(3):
            y = rt.all_reduce(x)
        torch.cuda.synchronize()
        out["healthy"] = bool(torch.all(y == want))

        def attempt(launch, mode):
            res = {"victim": rank == victim}
            dist.barrier()
            t0 = time.perf_counter()
            if rank != victim:
                launch()
                torch.cuda.synchronize()
                res["seconds"] = time.perf_counter() - t0
                report = rt.failure()
                res["detected"] = report is not None
                res["report"] = report or ""
            dist.barrier()  # the victim waits here on the host, not on the GPU
            rt.reset()
            y2 = rt.all_reduce(x)
            torch.cuda.synchronize()
            res["recovered"] = bool(torch.all(y2 == want)) and rt.failure() is None
            out[mode] = res

        attempt(lambda: rt.all_reduce(x), "eager")
        # graph mode: every rank captures; the victim does not replay
        g_out = torch.empty_like(x)
        stream = torch.cuda.Stream(device=device)
        stream.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream), rt.capture(stream=stream):
            rt.all_reduce(x, out=g_out)
        attempt(lambda: graph.replay(), "graph")
        del graph
        dist.barrier()
        rt.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        out["error"] = f"{type(exc).__name__}: {exc}"
    queue.put(out)


def run(world: int = 2, timeout_ms: int = 1000, victim: int = 1, port: int = 29677) -> dict:
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_child, args=(r, world, port, timeout_ms, victim, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.monotonic() + SETUP_TIMEOUT_S + 20 * timeout_ms / 1000 + 60
    for _ in procs:
        left = max(1.0, deadline - time.monotonic())
        try:
            results.append(queue.get(timeout=left))
        except Exception:  # noqa: BLE001
            break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.terminate()
    results.sort(key=lambda r: r["rank"])
    errs = [f"rank {r['rank']}: {r['error']}" for r in results if "error" in r]
    if len(results) != world:
        errs.append(f"only {len(results)} of {world} ranks reported")
    for r in results:
        if "error" not in r:
            errs += problems(r, timeout_ms)
    return {"world": world, "timeout_ms": timeout_ms, "victim": victim, "results": results, "problems": errs,
            "passed": not errs}


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--world", type=int, default=2, choices=(2, 4))
    parser.add_argument("--timeout-ms", type=int, default=1000)
    parser.add_argument("--victim", type=int, default=1)
    parser.add_argument("--port", type=int, default=29677)
    args = parser.parse_args(argv)
    result = run(args.world, args.timeout_ms, args.victim, args.port)
    print(json.dumps(result))
    return 0 if result["passed"] else 1


if __name__ == "__main__":
    sys.exit(main())
