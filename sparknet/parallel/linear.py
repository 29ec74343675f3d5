"""Column- and row-parallel linear layers for sequence-parallel prefill and decode.

Weights are stored K-major (``[out_features_shard, in_features]``), as the tcgen05
kernels read them.  In sequence-parallel prefill the activations between layers are
sharded by token:

* ``ColumnParallelLinear.forward(x_shard)`` = all_gather(x_shard) @ W_shard.T in one
  kernel (``AllReduce.ag_gemm``): copy CTAs push the shard while tensor cores start on
  local rows;
* ``RowParallelLinear.forward(a)`` = reduce_scatter(a @ W_shard.T) in one kernel
  (``AllReduce.gemm_rs``): tiles leave over NVLink from the epilogue.

For decode (a few tokens, replicated activations) ``RowParallelLinear.decode`` does
the local GEMM and the fused all-reduce + residual + RMSNorm.
"""

from __future__ import annotations

import torch


class ColumnParallelLinear:
    def __init__(self, weight_shard: torch.Tensor, runtime):
        if weight_shard.dim() != 2 or weight_shard.dtype != torch.bfloat16:
            raise ValueError("weight shard must be [out/W, in] bfloat16")
        self.weight = weight_shard.contiguous()
        self.runtime = runtime

    def forward(self, x_shard: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Sequence-parallel: all-gather the token shards and multiply, fused."""
        return self.runtime.ag_gemm(x_shard, self.weight, out=out)

    def decode(self, x: torch.Tensor) -> torch.Tensor:
        """Replicated activations: a local GEMM, no collective."""
        return x @ self.weight.T


class RowParallelLinear:
    def __init__(self, weight_shard: torch.Tensor, runtime):
        if weight_shard.dim() != 2 or weight_shard.dtype != torch.bfloat16:
            raise ValueError("weight shard must be [out, in/W] bfloat16")
        self.weight = weight_shard.contiguous()
        self.runtime = runtime

    def forward(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Sequence-parallel: multiply and reduce-scatter the partial sums by token, fused."""
        return self.runtime.gemm_rs(a, self.weight, out=out)

    def decode(self, a: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
               eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
        """Decode: local GEMM, then all-reduce + residual add + RMSNorm in one kernel."""
        partial = a @ self.weight.T
        return self.runtime.all_reduce_residual_rmsnorm(partial, residual, gamma, eps, residual_out=residual)


__all__ = ["ColumnParallelLinear", "RowParallelLinear"]
