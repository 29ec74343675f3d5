"""Device-side timing helpers: CUDA events on the launching stream, L2 flushing and
slowest-rank statistics (every multi-GPU number is the max over ranks)."""

from __future__ import annotations

import math
import statistics
from typing import Sequence

L2_FLUSH_BYTES = 256 * 1024 * 1024  # twice B200's 126 MB L2


class L2Flusher:
    """Writes a buffer larger than L2 so the next kernel starts cold."""

    def __init__(self, device, nbytes: int = L2_FLUSH_BYTES):
        import torch

        self.buf = torch.empty(nbytes // 4, dtype=torch.int32, device=device)

    def __call__(self) -> None:
        self.buf.fill_(0x5A5A5A5A)


def slowest_rank_median(per_rank: Sequence[Sequence[float]]) -> float:
    """Median over samples of the max over ranks (samples aligned by index)."""
    samples = [max(vals) for vals in zip(*per_rank)]
    return statistics.median(samples)


def geomean(values: Sequence[float]) -> float:
    values = [v for v in values if v and v > 0]
    return math.exp(sum(math.log(v) for v in values) / len(values)) if values else float("nan")
