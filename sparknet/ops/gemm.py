"""``C = A @ B.T`` on 5th-generation tensor cores (tcgen05, TMEM accumulators, TMA).

Both operands are K-major (row-major ``A[M, K]`` and ``B[N, K]``), bf16 in, fp32
accumulation, bf16 out.  K must be a multiple of 64 and N of 32.  Two kernels, both
persistent and warp-specialised (TMA warp, MMA warp, four epilogue warps) with a
double-buffered accumulator in TMEM:

* ``block_n="pair"`` (default): a CTA pair (``tcgen05.mma.cta_group::2``) per 256 x 256
  tile, each CTA staging 128 rows of A and 128 rows of B per K step, 6 stages; measured
  faster than the one-CTA kernel at every shape tried (8192 x 7168 x 8192: ~1460 against
  ~1425 TFLOP/s on one B200);
* ``block_n=256`` / ``128``: one CTA per 128 x ``block_n`` tile, 4 (6) stages.
"""

from __future__ import annotations

import torch

from .. import _native

_ERRORS = {1: "an mbarrier wait timed out", 2: "a peer flag wait timed out"}


class GemmError(RuntimeError):
    """A tcgen05 GEMM gave up on a bounded wait (its error word was set)."""
    pass


def _err_word(device) -> torch.Tensor:
    key = (device.type, device.index)
    buf = _err_word.cache.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=device)
        _err_word.cache[key] = buf
    return buf


_err_word.cache = {}


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, *, block_n: int | str = "pair",
         max_ctas: int = 0, check: bool = False) -> torch.Tensor:
    """``a @ b.T`` for bf16 ``a [M, K]`` and ``b [N, K]``."""
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise ValueError("gemm takes bfloat16 operands")
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError("a and b must share K")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    err = _err_word(a.device)
    if block_n == "pair":
        _native.load().gemm_pair(a, b, out, err, max_ctas // 2)
    else:
        _native.load().gemm(a, b, out, err, int(block_n), max_ctas)
    if check:
        torch.cuda.synchronize(a.device)
        code = int(err.item())
        if code:
            err.zero_()
            raise GemmError(f"tcgen05 GEMM failed: {_ERRORS.get(code, code)}")
    return out


__all__ = ["GemmError", "gemm"]
