"""Column- and row-parallel linear layers for sequence-parallel prefill and decode.

Weights are stored K-major (``[out_features_shard, in_features]``), as the tcgen05
kernels read them.  In sequence-parallel prefill the activations between layers are
sharded by token:

* ``ColumnParallelLinear.forward(x_shard)`` = all_gather(x_shard) @ W_shard.T in one
  kernel (``AllReduce.ag_gemm``): copy CTAs push the shard while tensor cores start on
  local rows;
* ``RowParallelLinear.forward(a)`` = reduce_scatter(a @ W_shard.T) in one kernel
  (``AllReduce.gemm_rs``): tiles leave over NVLink from the epilogue.

With ``fp8=True`` the weight is quantised once to e4m3 with one UE8M0 scale per
128 x 128 block, the activations per call with one scale per row and 128 columns, and
the block-scaled forms of the same kernels run (``ag_gemm_fp8`` / ``gemm_rs_fp8``):
half the NVLink bytes of the gather, bf16 output.

For decode (a few tokens, replicated activations) the local product is the tcgen05
decode GEMM (``sparknet.ops.decode_gemm``, 1..256 token rows, in_features a multiple
of 64; a torch matmul outside that range), and ``RowParallelLinear.decode`` follows it
with the fused all-reduce + residual + RMSNorm.
"""

from __future__ import annotations

from typing import Optional

import torch

DECODE_MAX_TOKENS = 256  # the decode GEMM's row limit
DECODE_K_MULTIPLE = 64


def _local_product(x: torch.Tensor, weight: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ weight.T`` for replicated decode activations."""
    if (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and 1 <= x.shape[0] <= DECODE_MAX_TOKENS
            and x.shape[1] % DECODE_K_MULTIPLE == 0 and x.stride(1) == 1):
        from sparknet.ops.decode_gemm import linear

        return linear(x, weight, out)
    if out is None:
        return x @ weight.T
    return torch.mm(x, weight.T, out=out)


class _ParallelLinear:
    def __init__(self, weight_shard: torch.Tensor, runtime, *, fp8: bool, what: str):
        if weight_shard.dim() != 2 or weight_shard.dtype != torch.bfloat16:
            raise ValueError(f"weight shard must be {what} bfloat16")
        self.weight = weight_shard.contiguous()
        self.runtime = runtime
        self.fp8 = bool(fp8)
        self.weight_q = self.weight_scales = None
        if self.fp8:
            if self.weight.shape[0] % 128 or self.weight.shape[1] % 128:
                raise ValueError("fp8 weights need both dimensions a multiple of 128 (128 x 128 scale blocks)")
            from sparknet.ops import fp8 as fp8_ops

            self.weight_q, self.weight_scales = fp8_ops.quantize_weight(self.weight)

    @staticmethod
    def _quantize(x: torch.Tensor):
        from sparknet.ops import fp8 as fp8_ops

        return fp8_ops.quantize_act(x.contiguous())


class ColumnParallelLinear(_ParallelLinear):
    """Output features sharded over ranks: weight ``[out/W, in]``."""

    def __init__(self, weight_shard: torch.Tensor, runtime, *, fp8: bool = False):
        super().__init__(weight_shard, runtime, fp8=fp8, what="[out/W, in]")

    def forward(self, x_shard: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sequence-parallel: all-gather the token shards and multiply, fused."""
        if self.fp8:
            xq, sx = self._quantize(x_shard)
            return self.runtime.ag_gemm_fp8(xq, sx, self.weight_q, self.weight_scales, out=out)
        return self.runtime.ag_gemm(x_shard, self.weight, out=out)

    def decode(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Replicated activations: a local GEMM, no collective."""
        return _local_product(x, self.weight, out)


class RowParallelLinear(_ParallelLinear):
    """Input features sharded over ranks: weight ``[out, in/W]``."""

    def __init__(self, weight_shard: torch.Tensor, runtime, *, fp8: bool = False):
        super().__init__(weight_shard, runtime, fp8=fp8, what="[out, in/W]")

    def forward(self, a: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sequence-parallel: multiply and reduce-scatter the partial sums by token, fused."""
        if self.fp8:
            aq, sa = self._quantize(a)
            return self.runtime.gemm_rs_fp8(aq, sa, self.weight_q, self.weight_scales, out=out)
        return self.runtime.gemm_rs(a, self.weight, out=out)

    def decode(self, a: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
               eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
        """Decode: local GEMM, then all-reduce + residual add + RMSNorm in one kernel
        (the new residual is written in place)."""
        partial = _local_product(a, self.weight)
        return self.runtime.all_reduce_residual_rmsnorm(partial, residual, gamma, eps, residual_out=residual)


__all__ = ["ColumnParallelLinear", "RowParallelLinear"]
