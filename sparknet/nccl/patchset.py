"""The NCCL patch series: empty on B200.

The reference ships four patches to NCCL 2.30.7 (an AArch64 acquire fence in the IB
transport and switchless-ring tuning; ``sparknet/nccl/patches/series`` of the
reference).  None applies to an x86 NVSwitch box, so NCCL runs as released and is the
unmodified baseline.  The functions keep the reference's interface so image builds
that call them keep working; ``export`` writes an empty series with a README.
"""

from __future__ import annotations

from pathlib import Path

README = ("No NCCL patches are applied on B200: NCCL runs unmodified over NVLink/NVSwitch and is the baseline "
          "that sparknet's kernels are measured against.\n")


def patch_directory() -> Path:
    """Where the series would live (this package; it ships no patch files)."""
    return Path(__file__).resolve().parent


def series() -> list[str]:
    """The NCCL patch series: empty, stock NCCL serves an NVSwitch box."""
    return []


def missing(directory: str | Path | None = None) -> list[str]:
    """Patches of the series that ``directory`` lacks: none, stock NCCL needs no series."""
    return []


def export(directory: str | Path) -> list[Path]:
    """Write the (empty) patch series and its README into ``directory``; returns the written paths."""
    out = Path(directory)
    out.mkdir(parents=True, exist_ok=True)
    (out / "series").write_text("")
    (out / "README.md").write_text(README)
    return [out / "series", out / "README.md"]


__all__ = ["export", "missing", "patch_directory", "series"]
