"""Process groups for tensor parallelism on one NVSwitch box.

``init_tp()`` reads the torchrun environment (RANK, WORLD_SIZE, LOCAL_RANK,
MASTER_*), binds the rank to its GPU, initialises torch.distributed with NCCL for
CUDA tensors and gloo for setup exchanges, and builds the NVLink runtime over the
gloo group.  The returned ``TPGroup`` carries both and closes them in order.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta
from typing import Any, Optional

import torch
import torch.distributed as dist


@dataclass
class TPGroup:
    rank: int
    world: int
    device: torch.device
    cpu_group: Any
    runtime: Any

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.cpu_group)
        if self.runtime is not None:
            self.runtime.close()
        dist.barrier(group=self.cpu_group)
        dist.destroy_process_group()


def init_tp(*, max_size: int = 8 << 20, max_gather_bytes: int = 16 << 20, timeout_s: int = 120,
            runtime: bool = True, policy=None) -> TPGroup:
    """Join the tensor-parallel group of this process (LOCAL_RANK's GPU): the default
    process group, a gloo group for the setup exchange and, with ``runtime=True``, the
    NVLink runtime."""
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=timeout_s), device_id=device)
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))
    rt: Optional[Any] = None
    if runtime:
        from sparknet.oneshot import AllReduce

        kw = {"policy": policy} if policy is not None else {}
        rt = AllReduce.from_exchange_group(exchange_group=cpu, device=device, max_size=max_size,
                                           max_gather_bytes=max_gather_bytes, **kw)
    return TPGroup(dist.get_rank(), dist.get_world_size(), device, cpu, rt)


__all__ = ["TPGroup", "init_tp"]
