"""Hand-written sm_100a ops: tcgen05 GEMM, the fused prefill collectives (all-gather ->
GEMM, GEMM -> reduce-scatter) and the fused decode all-reduce + RMSNorm."""

from .gemm import gemm

__all__ = ["gemm"]
