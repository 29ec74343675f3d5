"""Tensor-parallel prefill GEMMs fused with their collectives (tcgen05 + NVLink).

``ag_gemm(runtime, x_shard, w)``  = all_gather(x_shard, dim 0) @ w.T   (QKV, gate/up)
``gemm_rs(runtime, a, w)``        = reduce_scatter(a @ w.T, dim 0)     (O, down)
``ag_gemm_fp8`` / ``gemm_rs_fp8``   the same on block-scaled fp8 operands
                                   (``sparknet.ops.fp8.quantize_act`` / ``quantize_weight``)

Both run as one kernel launch on every rank (see ``csrc/gemm_tcgen05.cu``); the
unfused equivalents (NCCL collective + cuBLAS GEMM) are ``ag_gemm_reference`` and
``gemm_rs_reference`` for tests and baselines.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def ag_gemm(runtime, x_shard: torch.Tensor, w: torch.Tensor, **kw) -> torch.Tensor:
    """``all_gather(x_shard) @ w.T`` in one kernel through ``runtime`` (``AllReduce.ag_gemm``)."""
    return runtime.ag_gemm(x_shard, w, **kw)


def gemm_rs(runtime, a: torch.Tensor, w: torch.Tensor, **kw) -> torch.Tensor:
    """``reduce_scatter(a @ w.T)`` in one kernel through ``runtime`` (``AllReduce.gemm_rs``)."""
    return runtime.gemm_rs(a, w, **kw)


def ag_gemm_fp8(runtime, xq_shard: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                **kw) -> torch.Tensor:
    """The block-scaled fp8 form of :func:`ag_gemm` (``AllReduce.ag_gemm_fp8``)."""
    return runtime.ag_gemm_fp8(xq_shard, sx, wq, sw, **kw)


def gemm_rs_fp8(runtime, aq: torch.Tensor, sa: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
                **kw) -> torch.Tensor:
    """The block-scaled fp8 form of :func:`gemm_rs` (``AllReduce.gemm_rs_fp8``)."""
    return runtime.gemm_rs_fp8(aq, sa, wq, sw, **kw)


def ag_gemm_reference(x_shard: torch.Tensor, w: torch.Tensor, group=None) -> torch.Tensor:
    """The unfused baseline: an NCCL all-gather into a full tensor, then a cuBLAS GEMM."""
    world = dist.get_world_size(group)
    full = torch.empty((x_shard.shape[0] * world, x_shard.shape[1]), dtype=x_shard.dtype, device=x_shard.device)
    dist.all_gather_into_tensor(full, x_shard, group=group)
    return full @ w.T


def gemm_rs_reference(a: torch.Tensor, w: torch.Tensor, group=None) -> torch.Tensor:
    """The unfused baseline: a cuBLAS GEMM, then an NCCL reduce-scatter."""
    world = dist.get_world_size(group)
    partial = a @ w.T
    out = torch.empty((a.shape[0] // world, w.shape[0]), dtype=a.dtype, device=a.device)
    dist.reduce_scatter_tensor(out, partial, group=group)
    return out


__all__ = ["ag_gemm", "ag_gemm_fp8", "ag_gemm_reference", "gemm_rs", "gemm_rs_fp8", "gemm_rs_reference"]
