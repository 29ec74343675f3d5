"""Hand-written sm_100a ops: tcgen05 GEMM, the decode GEMM (few tokens, split-K, fused
SwiGLU), the fused prefill collectives (all-gather -> GEMM, GEMM -> reduce-scatter) and
the fused decode all-reduce + RMSNorm."""

from .decode_gemm import DecodeGemm, interleave_gate_up, linear, split_gate_up
from .gemm import gemm

__all__ = ["DecodeGemm", "gemm", "interleave_gate_up", "linear", "split_gate_up"]
