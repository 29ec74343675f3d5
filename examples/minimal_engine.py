#!/usr/bin/env python3
"""The smallest engine that uses the library the way a serving recipe should.

One process per GPU of one NVSwitch box, launched with the environment that
``sparknet topology render <gpumap.json> <box> --transport nvlink --profile nvlink``
prints::

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/minimal_engine.py

It initialises torch.distributed with NCCL for CUDA tensors and gloo for the setup
exchange, builds the NVLink runtime from the policy in the environment, prepares it
before any CUDA graph, runs a few tensor-parallel decode steps of a small Llama-shaped
model eagerly and from a captured graph (every all-reduce goes through the policy;
the residual add + RMSNorm epilogue is fused into the all-reduce), checks health after
each step's host sync, and freezes lazy resolution once warm.
(After the reference's ``examples/minimal_engine.py``.)
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from sparknet import oneshot  # noqa: E402
from sparknet.models import LlamaConfig, TPLlama  # noqa: E402
from sparknet.policy import NVLINK_POLICY, CollectivePolicy  # noqa: E402


def dispatch_all_reduce(runtime, policy, x: torch.Tensor, world: int) -> torch.Tensor:
    """The policy decides, every rank alike, from dtype, shape, byte size and world."""
    nbytes = x.numel() * x.element_size()
    backend = policy.all_reduce_backend(nbytes, str(x.dtype).replace("torch.", ""),
                                        contiguous=x.is_contiguous(), world=world)
    if backend != "nccl":
        return runtime.all_reduce(x, algorithm=backend if backend != "nvls" or runtime.has_multicast else None)
    out = x.clone()
    dist.all_reduce(out)
    return out


def main() -> None:
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group(backend="cpu:gloo,cuda:nccl", timeout=timedelta(seconds=120), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    cpu_group = dist.new_group(backend="gloo")  # the setup exchange; never the NCCL communicator

    env = dict(os.environ)
    policy = CollectivePolicy.from_environment(env) if env.get("SPARKNET_ALLREDUCE_CAPACITY_BYTES") else NVLINK_POLICY
    runtime = oneshot.AllReduce.from_exchange_group(exchange_group=cpu_group, device=device,
                                                    max_size=policy.all_reduce_capacity_bytes,
                                                    max_gather_bytes=policy.all_gather_shard_bytes, policy=policy)
    runtime.prepare((torch.bfloat16,), padded_gather=True)  # before any capture
    if rank == 0:
        print("runtime:", {k: runtime.stats()[k] for k in ("transport", "dispatch_max_bytes", "oneshot_max_bytes")})

    # 1. a policy-dispatched all-reduce of a 6-token, 8192-wide decode activation
    hidden = torch.full((6, 8192), rank + 1, dtype=torch.bfloat16, device=device)
    expected = float(world * (world + 1) // 2)
    out = dispatch_all_reduce(runtime, policy, hidden, world)
    torch.cuda.synchronize()
    runtime.check_health()
    assert torch.all(out == expected), "all-reduce mismatch"

    # 2. a small TP Llama decoding with the fused all-reduce + residual + RMSNorm
    cfg = LlamaConfig(hidden=2048, layers=4, heads=16, kv_heads=8, head_dim=128, ffn=4096, vocab=16384)
    model = TPLlama(cfg, rank=rank, world=world, device=device, batch=4, max_len=128, runtime=runtime)
    model.fill_prompt_cache(16)
    model.tokens.copy_(torch.arange(4, device=device))
    model.step_kernels()                       # eager step
    torch.cuda.synchronize()
    runtime.check_health()
    model.capture()                            # the same step as one CUDA graph
    tokens = []
    for _ in range(4):
        model.replay()
        torch.cuda.synchronize()               # the step's own host sync
        runtime.check_health()                 # fail-stop: raises if any rank's wait timed out
        tokens.append(model.tokens.tolist())
    everyone = [None] * world
    dist.all_gather_object(everyone, tokens, group=cpu_group)
    assert all(t == everyone[0] for t in everyone), "ranks sampled different tokens"

    oneshot.freeze_kernel_resolution("warm-up complete")  # any later lazy resolution is a bug
    if rank == 0:
        print("ok:", runtime.stats()["calls"], "tokens:", tokens[-1])
    model.release()
    torch.cuda.synchronize()
    dist.barrier(group=cpu_group)
    runtime.close()
    dist.barrier(group=cpu_group)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
