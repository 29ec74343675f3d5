"""Block-scaled fp8 for prefill GEMMs: e4m3 values with power-of-two (UE8M0) scales.

Activations get one scale per row and 128 columns (1 x 128), weights one per
128 x 128 block.  Scales are stored as 512-byte chunks per (128 rows, 128 columns),
in the order tcgen05.cp stages them into TMEM for ``kind::mxf8f6f4.block_scale``
MMAs (``csrc/fp8_quant.cu`` documents the byte layout); :func:`scales_to_dense`
expands them back for checks.

    xq, sx = quantize_act(x)          # x [M, K] bf16
    wq, sw = quantize_weight(w)       # w [N, K] bf16
    y = gemm_fp8(xq, sx, wq, sw)      # ~ x @ w.T, bf16

The fused tensor-parallel forms are ``AllReduce.ag_gemm_fp8`` and ``gemm_rs_fp8``.
"""

from __future__ import annotations

import torch

from .. import _native
from .gemm import _ERRORS, GemmError, _err_word


def scale_bytes(rows: int, k: int) -> int:
    """Bytes of the scale chunks of a ``rows x k`` matrix: 512 per 128 rows and 128 columns."""
    return ((rows + 127) // 128) * (k // 128) * 512


def _alloc(rows: int, k: int, device):
    q = torch.empty((rows, k), dtype=torch.float8_e4m3fn, device=device)
    sf = torch.zeros(scale_bytes(rows, k), dtype=torch.uint8, device=device)
    return q, sf


def quantize_act(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``[M, K]`` -> (e4m3 ``[M, K]``, scales) with one scale per row and 128 columns."""
    q, sf = _alloc(x.shape[0], x.shape[1], x.device)
    _native.load().fp8_quantize_rows(x, q, sf)
    return q, sf


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``[N, K]`` -> (e4m3 ``[N, K]``, scales) with one scale per 128 x 128 block."""
    q, sf = _alloc(w.shape[0], w.shape[1], w.device)
    _native.load().fp8_quantize_blocks(w, q, sf)
    return q, sf


def scale_exponents(sf: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """UE8M0 exponent byte ``[rows, k // 128]`` of every (row, 128-column block)."""
    kb = k // 128
    rb = (rows + 127) // 128
    chunk = sf[: rb * kb * 512].view(rb, kb, 32, 4, 4)            # [rb, kb, i, g, j] (row = 32 g + i)
    return chunk[..., 0].permute(0, 3, 2, 1).reshape(rb * 128, kb)[:rows]  # byte j = 0: the block's exponent


def scales_to_dense(sf: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """fp32 ``[rows, k // 128]`` scale 2^(e - 127) of every (row, 128-column block) (exact)."""
    e = scale_exponents(sf, rows, k).to(torch.int32) - 127
    return torch.ldexp(torch.ones(e.shape, dtype=torch.float32, device=e.device), e)


def dequantize(q: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    """fp32 values of an e4m3 matrix from its UE8M0 scale chunks (activation or weight layout)."""
    rows, k = q.shape
    s = scales_to_dense(sf, rows, k).repeat_interleave(128, dim=1)
    return q.float() * s


def gemm_fp8(aq: torch.Tensor, sfa: torch.Tensor, bq: torch.Tensor, sfb: torch.Tensor,
             out: torch.Tensor | None = None, *, check: bool = False) -> torch.Tensor:
    """``dequant(aq) @ dequant(bq).T`` on tcgen05 block-scaled MMAs, bf16 out."""
    M, N = aq.shape[0], bq.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=aq.device)
    err = _err_word(aq.device)
    _native.load().gemm_fp8(aq, sfa, bq, sfb, out, err, 0)
    if check:
        torch.cuda.synchronize(aq.device)
        code = int(err.item())
        if code:
            err.zero_()
            raise GemmError(f"tcgen05 fp8 GEMM failed: {_ERRORS.get(code, code)}")
    return out


__all__ = ["dequantize", "gemm_fp8", "quantize_act", "quantize_weight", "scale_bytes", "scale_exponents",
           "scales_to_dense"]
