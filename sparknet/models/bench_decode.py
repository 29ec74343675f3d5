"""Llama-3-70B-shaped tensor-parallel decode throughput (``bench.py --workload decode``).

Random-init bf16 weights of the 70B architecture (80 layers, hidden 8192, 64/8 heads,
head_dim 128, SwiGLU 28672, vocab 128256, RoPE theta 5e5) sharded over the N GPUs; a
1024-token prompt is represented by random KV-cache entries; each timed step decodes
one token for every sequence of the batch through one CUDA graph replay.  Device
timing: CUDA events around K replays, max over ranks.  End to end: every step copies
the batch's input tokens from pinned host memory, replays, and copies the sampled
tokens back.
"""

from __future__ import annotations

import os
import statistics
import time

import torch
import torch.distributed as dist

from .llama import LlamaConfig, TPLlama

PROMPT = 1024
GENERATE = 256


def run_decode_bench(args, rank, world, device, cpu_group):
    from sparknet import _native

    comm = os.environ.get("SPARKNET_DECODE_COMM", "sparknet")
    cfg = LlamaConfig.llama3_70b()
    if args.layers != cfg.layers:
        raise SystemExit("the decode benchmark runs the full 80-layer model; --layers only for smoke tests")
    batch = args.batch
    max_len = PROMPT + GENERATE + 16
    if args.steps + args.warmup + 2 > GENERATE:
        raise SystemExit(f"steps + warmup must stay below {GENERATE} generated tokens")
    runtime = None
    if world > 1 and comm == "sparknet":
        from sparknet.oneshot import AllReduce

        runtime = AllReduce.from_exchange_group(exchange_group=cpu_group, device=device,
                                                max_size=max(8 << 20, batch * cfg.hidden * 2 * 2))
        if getattr(args, "no_pdl", False):
            runtime.set_pdl(False)  # on by default: the fused all-reduce + norm launches during the GEMM before it
        runtime.prepare((torch.bfloat16,))
    t0 = time.perf_counter()
    model = TPLlama(cfg, rank=rank, world=world, device=device, batch=batch, max_len=max_len, comm=comm,
                    runtime=runtime, group=None, attention=getattr(args, "attention", "auto"))
    model.fill_prompt_cache(PROMPT)
    torch.cuda.synchronize()
    init_s = time.perf_counter() - t0
    model.tokens.copy_(torch.randint(0, cfg.vocab, (batch,), generator=torch.Generator().manual_seed(5)).to(device))
    dist.barrier(group=cpu_group)
    model.capture()
    for _ in range(args.warmup):
        model.replay()
    torch.cuda.synchronize()
    dist.barrier(group=cpu_group)
    from sparknet.utils.clocks import ClockSampler

    sampler = ClockSampler(list(range(world)), interval_ms=50).start() if rank == 0 else None
    time.sleep(0.3)  # nvidia-smi takes a moment to begin sampling
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier(group=cpu_group)
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_start()
    start.record()
    for _ in range(args.steps):
        model.replay()
    end.record()
    end.synchronize()
    if sampler:
        sampler.mark_end()
    dist.barrier(group=cpu_group)
    clocks = sampler.stop() if sampler else None
    ms = start.elapsed_time(end)
    per = [None] * world
    dist.all_gather_object(per, ms, group=cpu_group)
    ms_max = max(per)
    if runtime is not None:
        runtime.check_health()
    # end to end: pinned H2D of the step's tokens, replay, D2H of the sampled tokens
    host_in = torch.randint(0, cfg.vocab, (batch,), dtype=torch.int64).pin_memory()
    host_out = torch.empty(batch, dtype=torch.int64).pin_memory()
    e2e = []
    for _ in range(max(3, min(args.steps, 16))):
        dist.barrier(group=cpu_group)
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        model.tokens.copy_(host_in, non_blocking=True)
        model.replay()
        host_out.copy_(model.tokens, non_blocking=True)
        en.record()
        en.synchronize()
        e2e.append(st.elapsed_time(en))
    gathered = [None] * world
    dist.all_gather_object(gathered, e2e, group=cpu_group)
    e2e_ms = statistics.median(max(g[i] for g in gathered) for i in range(len(e2e)))
    model.release()
    torch.cuda.synchronize()
    tok_s = batch * args.steps / (ms_max / 1000.0)
    return {
        "metric": "bf16 all-reduce p50 µs (max over ranks) @10K–2MiB, 2/4/8 B200; TP8 decode tok/s",
        "workload": "decode",
        "value": round(tok_s, 2),
        "unit": "tokens/s (whole job)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: random-init weights, random KV cache for a 1024-token prompt, random tokens",
        "config": {"model": "Llama-3-70B-shaped (80 layers, hidden 8192, 64/8 heads, FFN 28672, vocab 128256)",
                   "global_batch": batch, "seq_len": PROMPT, "parallelism": f"tp{world}", "comm": comm,
                   "gemm": model.gemm, "programmatic_dependent_launch": model.pdl,
                   "collective_pdl": bool(runtime.pdl) if runtime is not None else False,
                   "attention": model.attention,

                   "l2": "weights per step far exceed L2 (126 MB)"},
        "gpu_launches": model.launches_per_step() * args.steps,
        "clocks": clocks,
        "init_s": round(init_s, 1),
        "e2e": {"value": round(batch / (e2e_ms / 1000.0), 2), "unit": "tokens/s, pinned H2D tokens + replay + D2H",
                "h2d_bytes_per_step": batch * 8, "d2h_bytes_per_step": batch * 8,
                "api": "sparknet.models.TPLlama.replay"},
        "native_extension": _native.loaded_path(),
    }
