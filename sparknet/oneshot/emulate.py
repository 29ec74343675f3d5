"""Every rank of a collective inside one GPU (testing and single-GPU benchmarking).

``EmulatedGroup(world, device)`` holds ``world`` symmetric regions in one device
allocation; each collective is one cooperative launch whose ``blockIdx.y`` is the
rank, running exactly the device code the multi-process runtime runs.  Ranks that
wait on one another are thereby always co-resident (the cooperative launch
guarantees it), which separate processes sharing one GPU could not promise.
"""

from __future__ import annotations

from typing import Sequence

import torch

from .. import _native
from .runtime import ALGO_CODES, GATHER_CODES, LL_CAP, PACK_BYTES, align_up


class EmulatedGroup:
    """Every rank of a group on one GPU: ``world`` regions and one cooperative launch per
    collective (rank = blockIdx.y), running the production protocol code; the protocol
    tests' group."""

    def __init__(self, world: int, device: torch.device | int | str = "cuda", *, max_size: int = 8 << 20,
                 max_gather_bytes: int = 4 << 20, timeout_ms: int = 2000):
        self.world = int(world)
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        C = _native.load()
        lam = align_up(max(max_size, 2 * max_size // self.world + 4096), 4096)
        self.caps = (lam, align_up(min(LL_CAP, max_gather_bytes), 4096), align_up(max_gather_bytes, 4096))
        with torch.cuda.device(self.device):
            self.comm = C.Comm(0, self.world, self.device.index, *self.caps, [], 0, 0, 0, True)
            self.comm.init_region()
            self.comm.set_timeout_us(int(timeout_ms) * 1000)

    def failures(self) -> list[dict]:
        return [dict(self.comm.status(r)) for r in range(self.world) if self.comm.failed_seq(r)]

    def check(self) -> None:
        bad = self.failures()
        if bad:
            raise RuntimeError(f"emulated collective failed: {bad}")

    def reset(self) -> None:
        torch.cuda.synchronize(self.device)
        self.comm.init_region()

    def all_reduce(self, inputs: Sequence[torch.Tensor], algorithm: str = "oneshot",
                   outs: Sequence[torch.Tensor] | None = None, blocks: int = 0, threads: int = 512):
        outs = [torch.empty_like(x) for x in inputs] if outs is None else list(outs)
        with torch.cuda.device(self.device):
            self.comm.all_reduce(list(inputs), outs, ALGO_CODES[algorithm], threads, blocks)
        return outs

    def reduce_scatter(self, inputs: Sequence[torch.Tensor]):
        rows = inputs[0].shape[0] // self.world
        outs = [torch.empty((rows, *x.shape[1:]), dtype=x.dtype, device=x.device) for x in inputs]
        chunk = outs[0].numel() * outs[0].element_size()
        with torch.cuda.device(self.device):
            self.comm.reduce_scatter(list(inputs), outs, chunk, chunk)
        return outs

    def all_gather(self, inputs: Sequence[torch.Tensor], dim: int = 0, algorithm: str = "ll"):
        x = inputs[0]
        dim = dim + x.dim() if dim < 0 else dim
        shape = list(x.shape)
        shape[dim] *= self.world
        outs = [torch.empty(shape, dtype=x.dtype, device=x.device) for _ in inputs]
        nbytes = x.numel() * x.element_size()
        if dim == 0:
            row, row_stride, src_stride = 0, 0, nbytes
        else:
            row = x.shape[-1] * x.element_size()
            row_stride, src_stride = row * self.world, row
        with torch.cuda.device(self.device):
            self.comm.all_gather(list(inputs), outs, nbytes, row, row_stride, src_stride, GATHER_CODES[algorithm])
        return outs

    def exchange(self, chunks: Sequence[torch.Tensor], copy_self: bool = False, fill: float = 0.0):
        parts = [torch.full_like(c, fill) for c in chunks]
        elem = chunks[0].element_size()
        chunk_bytes = chunks[0][0].numel() * elem
        with torch.cuda.device(self.device):
            self.comm.exchange(list(chunks), parts, chunk_bytes, chunks[0].stride(0) * elem,
                               parts[0].stride(0) * elem, 0, -1, copy_self)
        return parts

    def fused_norm(self, inputs, residuals, gamma, eps=1e-5, algorithm="oneshot", cluster=8, *,
                   max_clusters: int = 0, threads: int = 0):
        """Fused all-reduce + residual add + RMSNorm on every emulated rank.

        ``cluster`` CTAs share a row; ``max_clusters`` caps the clusters per rank (0:
        one per row up to the co-resident limit; fewer makes each cluster loop over
        rows); ``threads`` forces the block size (0: one 16-byte pack per thread)."""
        outs = [torch.empty_like(x) for x in inputs]
        res_outs = [torch.empty_like(x) for x in residuals]
        with torch.cuda.device(self.device):
            self.comm.fused_norm(list(inputs), list(residuals), gamma, float(eps), outs, res_outs,
                                 ALGO_CODES[algorithm], cluster, max_clusters, threads)
        return outs, res_outs

    def barrier(self, blocks: int = 1) -> None:
        with torch.cuda.device(self.device):
            self.comm.barrier(blocks)


__all__ = ["EmulatedGroup", "PACK_BYTES"]
