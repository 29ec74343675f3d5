"""Decode GEMM: ``x @ w.T`` for a few token rows on tcgen05 tensor cores.

``w`` is in ``nn.Linear`` layout ``[out_features, in_features]`` (bf16, K-major) and
``x`` is ``[tokens, in_features]`` with 1..256 tokens.  The kernel (``csrc/gemm_skinny.cu``)
streams the weight through TMA into 128-row tiles that are the MMA's M side, splits K
so one wave covers the GPU, and sums the split partials of a tile inside a thread-block
cluster through distributed shared memory, in a fixed order (no global scratch).

``swiglu=True`` fuses the SwiGLU activation: ``w`` is a gate/up weight in the
interleaved layout :func:`interleave_gate_up` builds ([64 gate rows; 64 up rows] per
128-row tile) and the result is ``silu(x @ gate.T) * (x @ up.T)`` of width
``out_features / 2``, with no intermediate tensor.

With ``pdl=True`` the launch uses programmatic dependent launch: the kernel may start
while the previous kernel on the stream is finishing and streams its first weight tiles
before it waits for that kernel's results (weights never depend on it).
"""

from __future__ import annotations

import torch

from .. import _native

INTERLEAVE_ROWS = 64


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``[F, K]`` gate and up weights -> ``[2F, K]`` with [64 gate; 64 up] row tiles."""
    if gate.shape != up.shape or gate.shape[0] % INTERLEAVE_ROWS:
        raise ValueError("gate and up must have the same shape with rows a multiple of 64")
    F, K = gate.shape
    t = F // INTERLEAVE_ROWS
    return torch.stack((gate.reshape(t, INTERLEAVE_ROWS, K), up.reshape(t, INTERLEAVE_ROWS, K)), 1).reshape(2 * F, K)


def split_gate_up(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of :func:`interleave_gate_up`."""
    F2, K = w.shape
    v = w.reshape(F2 // (2 * INTERLEAVE_ROWS), 2, INTERLEAVE_ROWS, K)
    return v[:, 0].reshape(F2 // 2, K), v[:, 1].reshape(F2 // 2, K)


class DecodeGemm:
    """The decode GEMM on one device (holds the error word)."""

    def __init__(self, device, max_splits: int = 0, pdl: bool = False):
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.C = _native.load()
        self.max_splits = int(max_splits)
        self.pdl = bool(pdl)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def __call__(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, *,
                 swiglu: bool = False) -> torch.Tensor:
        M = x.shape[0]
        N = w.shape[0]
        if out is None:
            out = torch.empty((M, N // 2 if swiglu else N), dtype=torch.bfloat16, device=x.device)
        self.C.skinny_gemm(x, w, out, self.err, 1 if swiglu else 0, self.max_splits, self.pdl)
        return out

    def qkv_rope(self, x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 positions: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 hq: int, hkv: int) -> None:
        """Decode QKV projection with RoPE and the KV-cache write in the epilogue.

        ``w`` is ``[(hq + 2 hkv) * 128, K]`` (q heads, then k heads, then v heads);
        rotated q goes to ``q_out [M, hq, 128]``, rotated k and plain v to
        ``k_cache`` / ``v_cache [M, lmax, hkv, 128]`` at ``positions [M]`` (int32);
        ``cos`` / ``sin`` are ``[lmax, 64]`` float32 (rotate-half form)."""
        self.C.skinny_qkv_rope(x, w, cos, sin, positions, q_out, k_cache, v_cache, self.err, hq, hkv, self.pdl)

    def check(self) -> None:
        torch.cuda.synchronize(self.device)
        code = int(self.err.item())
        if code:
            self.err.zero_()
            raise RuntimeError(f"decode GEMM failed: error {code} (an mbarrier wait timed out)")


_default: dict = {}


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, *, swiglu: bool = False) -> torch.Tensor:
    """``x @ w.T`` (or the fused SwiGLU of an interleaved gate/up weight) for decode."""
    key = x.device.index
    op = _default.get(key)
    if op is None:
        op = _default[key] = DecodeGemm(x.device)
    return op(x, w, out, swiglu=swiglu)


def plan(m: int, n: int, k: int, sms: int = 148, max_splits: int = 0) -> dict:
    """The launch the kernel would use: token padding, stages, splits, tiles, shared memory."""
    mp, stages, splits, kb, tiles, smem = _native.load().skinny_plan(m, n, k, sms, max_splits)
    return {"mma_n": mp, "stages": stages, "splits": splits, "k_blocks_per_split": kb, "tiles": tiles,
            "smem_bytes": smem, "ctas": splits * tiles}


__all__ = ["DecodeGemm", "interleave_gate_up", "linear", "plan", "split_gate_up", "INTERLEAVE_ROWS"]
