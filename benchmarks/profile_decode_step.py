#!/usr/bin/env python3
"""One rank's share of a Llama-3-70B TP decode step on one GPU, for kernel profiles.

Builds the shard a TP``--tp`` rank holds (hidden 8192, 64/tp query heads, 8/tp KV
heads, FFN 28672/tp, vocab 128256/tp) with ``--layers`` layers, fills a 1024-token KV
cache, warms up, then runs ``--steps`` eager decode steps.  With world size 1 the
all-reduce epilogue is the local add+RMSNorm kernel, so a profiler sees every other
kernel of a step exactly as a TP rank runs it.  Run under ncu with a launch filter,
e.g. ``ncu --metrics gpu__time_duration.sum --clock-control none -s <warm-up launches>
-c <launches> python benchmarks/profile_decode_step.py --layers 4 --steps 1``.
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from sparknet.models.llama import LlamaConfig, TPLlama  # noqa: E402


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--graph", action="store_true", help="time graph replays instead of eager steps")
    ap.add_argument("--gemm", choices=["sparknet", "cublas"], default="sparknet")
    ap.add_argument("--attention", choices=["auto", "simt", "tcgen05"], default="auto")
    args = ap.parse_args()
    t = args.tp
    cfg = LlamaConfig(hidden=8192, layers=args.layers, heads=64 // t, kv_heads=max(1, 8 // t), head_dim=128,
                      ffn=28672 // t, vocab=128256 // t)
    device = torch.device("cuda", 0)
    model = TPLlama(cfg, rank=0, world=1, device=device, batch=args.batch, max_len=1280 + 16, gemm=args.gemm,
                    attention=args.attention)
    model.fill_prompt_cache(1024)
    for _ in range(args.warmup):
        model.step_kernels()
    torch.cuda.synchronize()
    if args.graph:
        model.capture()
        run = model.replay
    else:
        run = model.step_kernels
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    st.record()
    for _ in range(args.steps):
        run()
    en.record()
    en.synchronize()
    ms = st.elapsed_time(en) / args.steps
    per_layer = ms / args.layers
    weights = sum(v.numel() * 2 for L in model.layers for k, v in L.items() if k.startswith("w")) / args.layers
    print(f"step {ms:.3f} ms ({per_layer * 1000:.1f} us/layer, {weights / (per_layer / 1000) / 1e12:.2f} TB/s of "
          f"layer weights), wall {1000 * (time.perf_counter() - t0) / args.steps:.3f} ms")
    return 0


if __name__ == "__main__":
    sys.exit(main())
