"""Transport protocol and geometry of the NVLink collectives (after the reference's
``sparknet/transport/base.py:10-86``, where the seam separated the GPU protocol from
the RDMA posting side).

On an NVSwitch box the GPU protocol posts its own stores, so a transport's job is the
region lifecycle: allocate this rank's symmetric region, describe it to peers
(``local_blob``), map every peer's region (``connect``), expose the mapped base
addresses (and, for NVLS, the multicast alias), report fail-stop state and release
everything.  The runtime calls them in that order.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional, Protocol, runtime_checkable

MAX_RANKS = 8


@dataclass(frozen=True)
class Geometry:
    """What a transport needs to build the regions; identical on every rank except ``rank``."""

    world_size: int
    rank: int
    device_index: int
    region_bytes: int
    multicast_bytes: int = 0

    def validate(self) -> list[str]:
        problems = []
        if not 1 <= self.world_size <= MAX_RANKS:
            problems.append(f"world_size must be 1..{MAX_RANKS}")
        if not 0 <= self.rank < self.world_size:
            problems.append("rank must belong to the group")
        if self.device_index < 0:
            problems.append("device_index must be a CUDA device ordinal")
        if self.region_bytes <= 0 or self.region_bytes % 4096:
            problems.append("region_bytes must be a positive multiple of 4096")
        if self.multicast_bytes < 0 or self.multicast_bytes % 4096:
            problems.append("multicast_bytes must be a non-negative multiple of 4096")
        return problems


@dataclass(frozen=True)
class TransportCapability:
    """What a transport can do on this host, decided without touching the fabric."""

    name: str
    available: bool
    reasons: tuple[str, ...] = ()
    details: dict[str, Any] = field(default_factory=dict)


@runtime_checkable
class Transport(Protocol):
    """How a runtime reaches its peers' memory: connect over the exchange group, then every
    rank's region base and the optional multicast alias."""
    name: str
    world_size: int
    rank: int

    def local_blob(self) -> bytes: ...
    def connect(self, group) -> None: ...
    def start(self) -> None: ...
    def stop(self) -> None: ...
    def bases(self) -> list[int]: ...
    def multicast(self) -> Optional[tuple[int, int, int]]: ...
    def failed(self) -> bool: ...
    def error(self) -> str: ...
    def stats(self) -> dict[str, Any]: ...
    def close(self) -> None: ...


__all__ = ["MAX_RANKS", "Geometry", "Transport", "TransportCapability"]
