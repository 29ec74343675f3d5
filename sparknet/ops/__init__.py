"""Hand-written sm_100a ops: tcgen05 GEMM (bf16 and block-scaled fp8), the decode GEMM
(few tokens, split-K, fused SwiGLU / RoPE epilogues), the fused prefill collectives
(all-gather -> GEMM, GEMM -> reduce-scatter), split-KV decode attention and the fused
decode all-reduce + RMSNorm."""

from .attention import decode_attention
from .decode_gemm import DecodeGemm, interleave_gate_up, linear, split_gate_up
from .gemm import gemm
from .prefill import ag_gemm, ag_gemm_fp8, ag_gemm_reference, gemm_rs, gemm_rs_fp8, gemm_rs_reference

__all__ = ["DecodeGemm", "ag_gemm", "ag_gemm_fp8", "ag_gemm_reference", "gemm", "gemm_rs", "gemm_rs_fp8",
           "gemm_rs_reference",
           "decode_attention", "interleave_gate_up", "linear", "split_gate_up"]
