#!/usr/bin/env python3
"""Run one sparknet kernel on one GPU, timed with CUDA events, for kernel profiles.

    python benchmarks/profile_kernels.py allreduce --world 8 --bytes 2097152
    python benchmarks/profile_kernels.py fused_norm --world 8 --tokens 32
    python benchmarks/profile_kernels.py allgather --world 8 --bytes 491520
    python benchmarks/profile_kernels.py gemm --m 8192 --n 7168 --k 8192
    python benchmarks/profile_kernels.py attention --batch 8 --heads 8 --kv-heads 1 --length 1024
    python benchmarks/profile_kernels.py decode_gemm --m 8 --n 7168 --k 8192 --swiglu

Collectives run through ``EmulatedGroup``: every rank of the collective is one
``blockIdx.y`` slice of a single cooperative launch on this GPU, running the same
device code a multi-process rank runs (so a profile sees all ranks' traffic at once:
per-rank figures are the totals divided by the world size).  Each case does
``--warmup`` untimed launches, then ``--iters`` launches each timed by CUDA events on
the launching stream, with a 256 MiB L2 flush between them outside the events, and
prints one JSON line with the median and the algorithmic bytes or FLOPs.  Under ncu,
capture with ``-k regex:<kernel> -s <warmup> -c 1``.
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def _time(fn, warmup: int, iters: int, device) -> list[float]:
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    out = []
    for _ in range(iters):
        flush.fill_(1)
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        st.record()
        fn()
        en.record()
        en.synchronize()
        out.append(st.elapsed_time(en) * 1000.0)
    return out


def _gemm_stamps(x, w, y, swiglu, device) -> dict:
    """Phase timing of one cold decode-GEMM launch from per-CTA %globaltimer stamps:
    entry (relative to the first CTA's), set-up, first data, streaming, MMA drain, park
    + cluster barrier, reduce; p50 / max over CTAs in µs."""
    C = _native_mod()
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    info = C.skinny_plan(x.shape[0], w.shape[0], x.shape[1], sms, 0)
    ctas = info[2] * info[4]
    st = torch.zeros(ctas * 8, dtype=torch.int64, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    flush.fill_(1)
    torch.cuda.synchronize(device)
    C.skinny_gemm(x, w, y, err, 1 if swiglu else 0, 0, False, st)
    torch.cuda.synchronize(device)
    t = st.view(ctas, 8).double().cpu() / 1000.0
    t0 = t[:, 0].min()
    names = ["entry", "setup", "wait_prev", "first_data", "stream", "mma_drain", "park_sync", "reduce_exit"]
    out = {}
    for i, n in enumerate(names):
        d = (t[:, 0] - t0) if i == 0 else (t[:, i] - t[:, i - 1])
        out[n] = {"p50": round(float(d.median()), 2), "max": round(float(d.max()), 2)}
    out["span"] = round(float(t[:, 7].max() - t0), 2)
    return out


def _native_mod():
    from sparknet import _native

    return _native.load()


def _time_graph(fns, reps: int, device) -> float:
    """Microseconds per call: one CUDA graph of every fn in ``fns`` (each touching its
    own inputs, together larger than L2, so every call reads cold data), replayed
    ``reps`` times after one warm-up replay."""
    for fn in fns:
        fn()
    torch.cuda.synchronize(device)
    stream = torch.cuda.Stream(device=device)
    stream.wait_stream(torch.cuda.current_stream(device))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for fn in fns:
            fn()
    g.replay()
    torch.cuda.synchronize(device)
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(reps):
        g.replay()
    en.record()
    en.synchronize()
    return st.elapsed_time(en) * 1000.0 / (reps * len(fns))


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("kernel", choices=["allreduce", "fused_norm", "allgather", "reduce_scatter", "gemm", "gemm_fp8",
                                       "attention", "decode_gemm", "cublas_decode_gemm"])
    ap.add_argument("--swiglu", action="store_true", help="decode_gemm: fused SwiGLU epilogue")
    ap.add_argument("--tune", type=int, default=0, metavar="CTAS_PER_SM",
                    help="decode_gemm: skinny_tune(ctas_per_sm) before running (0 = default)")
    ap.add_argument("--pdl", action="store_true", help="decode_gemm: programmatic dependent launch")
    ap.add_argument("--impl", type=int, default=0, choices=(0, 1, 2),
                    help="attention: 0 tensor cores where eligible, 1 CUDA cores, 2 tensor cores")
    ap.add_argument("--stamps", action="store_true",
                    help="decode_gemm, attention --impl 2: per-CTA %%globaltimer phase stamps of one cold launch "
                         "(µs percentiles)")
    ap.add_argument("--world", type=int, default=8)
    ap.add_argument("--bytes", type=int, default=2 << 20, help="bytes per rank (collectives)")
    ap.add_argument("--algorithm", default="", help="oneshot/twoshot (all-reduce, fused norm), ll/push (gather)")
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=7168)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--block-n", type=lambda v: v if v == "pair" else int(v), default="pair",
                    help="gemm: 256, 128 or pair (a CTA pair per 256 x 256 tile)")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--kv-heads", type=int, default=1)
    ap.add_argument("--length", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device).manual_seed(0)
    row = {"kernel": args.kernel}

    if args.kernel in ("allreduce", "fused_norm", "allgather", "reduce_scatter"):
        from sparknet.oneshot.emulate import EmulatedGroup

        W = args.world
        g = EmulatedGroup(W, device, max_size=max(8 << 20, args.bytes), max_gather_bytes=max(4 << 20, args.bytes))
        if args.kernel == "fused_norm":
            H, T = args.hidden, args.tokens
            xs = [torch.randn(T, H, generator=gen, device=device).bfloat16() for _ in range(W)]
            rs = [torch.randn(T, H, generator=gen, device=device).bfloat16() for _ in range(W)]
            gamma = (1 + 0.02 * torch.randn(H, generator=gen, device=device)).bfloat16()
            algo = args.algorithm or "oneshot"
            fn = lambda: g.fused_norm(xs, rs, gamma, algorithm=algo)  # noqa: E731
            row.update(world=W, tokens=T, hidden=H, algorithm=algo, bytes_per_rank=T * H * 2)
        else:
            n = args.bytes // 2
            xs = [torch.randn(n, generator=gen, device=device).bfloat16() for _ in range(W)]
            if args.kernel == "allreduce":
                algo = args.algorithm or "oneshot"
                outs = [torch.empty_like(x) for x in xs]
                fn = lambda: g.all_reduce(xs, algorithm=algo, outs=outs)  # noqa: E731
            elif args.kernel == "allgather":
                algo = args.algorithm or "ll"
                fn = lambda: g.all_gather(xs, algorithm=algo)  # noqa: E731
            else:
                algo = "lamport"
                fn = lambda: g.reduce_scatter(xs)  # noqa: E731
            row.update(world=W, bytes_per_rank=args.bytes, algorithm=algo)
        samples = _time(fn, args.warmup, args.iters, device)
        g.check()
    elif args.kernel == "gemm":
        from sparknet.ops.gemm import gemm

        M, N, K = args.m, args.n, args.k
        a = torch.randn(M, K, generator=gen, device=device).bfloat16()
        b = (0.02 * torch.randn(N, K, generator=gen, device=device)).bfloat16()
        c = torch.empty(M, N, dtype=torch.bfloat16, device=device)
        fn = lambda: gemm(a, b, c, block_n=args.block_n)  # noqa: E731
        samples = _time(fn, args.warmup, args.iters, device)
        gemm(a, b, c, block_n=args.block_n, check=True)
        row.update(m=M, n=N, k=K, block_n=args.block_n, flops=2 * M * N * K)
        row["tflops"] = 2 * M * N * K / (statistics.median(samples) * 1e-6) / 1e12
    elif args.kernel == "gemm_fp8":
        from sparknet.ops import fp8

        M, N, K = args.m, args.n, args.k
        xq, sx = fp8.quantize_act(torch.randn(M, K, generator=gen, device=device).bfloat16())
        wq, sw = fp8.quantize_weight((0.02 * torch.randn(N, K, generator=gen, device=device)).bfloat16())
        c = torch.empty(M, N, dtype=torch.bfloat16, device=device)
        fn = lambda: fp8.gemm_fp8(xq, sx, wq, sw, c)  # noqa: E731
        samples = _time(fn, args.warmup, args.iters, device)
        fp8.gemm_fp8(xq, sx, wq, sw, c, check=True)
        row.update(m=M, n=N, k=K, flops=2 * M * N * K)
        row["tflops"] = 2 * M * N * K / (statistics.median(samples) * 1e-6) / 1e12
    elif args.kernel in ("decode_gemm", "cublas_decode_gemm"):
        from sparknet.ops.decode_gemm import DecodeGemm, plan

        M, N, K = args.m, args.n, args.k
        x = torch.randn(M, K, generator=gen, device=device).bfloat16()
        copies = max(1, -(-(400 << 20) // (N * K * 2)))  # > 3x L2 of weights in the graph
        ws = [(0.02 * torch.randn(N, K, generator=gen, device=device)).bfloat16() for _ in range(copies)]
        w = ws[0]
        if args.kernel == "decode_gemm":
            if args.tune:
                _native_mod().skinny_tune(args.tune)
                row["tune"] = args.tune
            op = DecodeGemm(device, pdl=args.pdl)
            row["pdl"] = args.pdl
            y = op(x, w, swiglu=args.swiglu)
            fn = lambda: op(x, w, y, swiglu=args.swiglu)  # noqa: E731
            fns = [lambda w=w: op(x, w, y, swiglu=args.swiglu) for w in ws]
            row.update(plan(M, N, K, torch.cuda.get_device_properties(device).multi_processor_count))
        else:
            y = torch.empty(M, N, dtype=torch.bfloat16, device=device)
            fn = lambda: torch.mm(x, w.t(), out=y)  # noqa: E731
            fns = [lambda w=w: torch.mm(x, w.t(), out=y) for w in ws]
        samples = _time(fn, args.warmup, args.iters, device)
        row["graph_us"] = _time_graph(fns, 20, device)
        if args.kernel == "decode_gemm":
            op.check()
            if args.stamps:
                row["phases_us"] = _gemm_stamps(x, ws[-1], y, args.swiglu, device)
        row.update(m=M, n=N, k=K, swiglu=args.swiglu, weight_bytes=N * K * 2, copies=copies)
        row["weight_tbs"] = N * K * 2 / (row["graph_us"] * 1e-6) / 1e12
    else:
        from sparknet import _native

        C = _native.load()
        B, Hq, Hkv, L, D = args.batch, args.heads, args.kv_heads, args.length, 128
        Lmax = L + 64
        q = torch.randn(B, Hq, D, generator=gen, device=device).bfloat16()
        k = torch.randn(B, Lmax, Hkv, D, generator=gen, device=device).bfloat16()
        v = torch.randn(B, Lmax, Hkv, D, generator=gen, device=device).bfloat16()
        lengths = torch.full((B,), L, dtype=torch.int32, device=device)
        out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=device)
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        ws = torch.zeros(C.attention_workspace_floats(B, Hq, Hkv, Lmax, sms), dtype=torch.float32, device=device)
        def attend(kk, vv):
            C.decode_attention(q, kk, vv, lengths, out, ws, Lmax, D ** -0.5, False, args.impl)

        if args.stamps and args.impl == 2:
            # one cold launch with per-CTA phase stamps (tensor-core kernel)
            nsplit = -(-Lmax // (128 if Lmax <= 64 * 128 else 256))
            st = torch.zeros(B * Hkv * nsplit * 12, dtype=torch.int64, device=device)
            flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
            flush.fill_(1)
            torch.cuda.synchronize(device)
            C.decode_attention(q, k, v, lengths, out, ws, Lmax, D ** -0.5, False, 2, st)
            torch.cuda.synchronize(device)
            t = st.view(-1, 12).double().cpu() / 1000.0
            t = t[t[:, 0] > 0]  # CTAs of the launch (the buffer is sized for the largest split)
            t0 = t[:, 0].min()
            names = ["entry", "setup", "issue_q_len", "first_k", "scores", "softmax", "output", "partial_count",
                     "merge_ml", "merge_weights", "merge_sum", "merge_out"]  # cluster merge: 7 = parked, 11 = merged
            phases = {}
            prev = None
            for i, n in enumerate(names):
                col = t[:, i]
                ok = col > 0
                if i == 0:
                    d = col - t0
                else:
                    d = (col - prev)[ok & (prev > 0)]
                if d.numel():
                    phases[n] = {"p50": round(float(d.median()), 2), "max": round(float(d.max()), 2),
                                 "ctas": int(d.numel())}
                prev = torch.where(ok, col, prev) if prev is not None else col
            phases["span"] = round(float(t.max() - t0), 2)
            row["phases_us"] = phases
        fn = lambda: attend(k, v)  # noqa: E731
        samples = _time(fn, args.warmup, args.iters, device)
        kv_bytes = 2 * B * Hkv * L * D * 2
        copies = max(1, min(64, -(-(400 << 20) // kv_bytes)))
        kvs = [(k, v)] + [(torch.randn_like(k), torch.randn_like(v)) for _ in range(copies - 1)]
        fns = [lambda kk=kk, vv=vv: attend(kk, vv) for kk, vv in kvs]
        row["graph_us"] = _time_graph(fns, 20, device)
        row.update(batch=B, heads=Hq, kv_heads=Hkv, length=L, kv_bytes=kv_bytes, copies=copies,
                   variant={0: "auto", 1: "simt", 2: "tcgen05"}[args.impl])
    med = statistics.median(samples)
    row.update(median_us=med, min_us=min(samples), iters=len(samples))
    if "bytes_per_rank" in row:
        row["per_rank_bytes_per_us"] = row["bytes_per_rank"] / med
    if "kv_bytes" in row:
        row["kv_gbs"] = row["kv_bytes"] / row["graph_us"] / 1e3
    print(json.dumps(row), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
