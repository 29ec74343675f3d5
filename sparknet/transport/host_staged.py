"""A host-memory test double of the transport seam (CPU only).

Regions are POSIX shared-memory segments named per rank; ``connect`` maps every
peer's segment by name through the caller's process group.  It keeps the seam's call
order and region sharing testable with gloo ranks on a machine without a GPU (what a
rank writes into a peer's mapped region, the peer reads), the way the reference's
simulator stands in for RDMA.
"""

from __future__ import annotations

import json
import os
import uuid
from multiprocessing import shared_memory
from typing import Any, Optional

from .base import Geometry, TransportCapability


def host_staged_capability() -> TransportCapability:
    """Whether the host-staged test transport can run here (``/dev/shm``)."""
    return TransportCapability(name="host-staged", available=os.path.isdir("/dev/shm"),
                               reasons=() if os.path.isdir("/dev/shm") else ("/dev/shm missing",))


class HostStagedTransport:
    """A CPU test double of the transport: regions in shared host memory, no GPU."""
    name = "host-staged"

    def __init__(self, geometry: Geometry):
        problems = geometry.validate()
        if problems:
            raise ValueError("; ".join(problems))
        self.geometry = geometry
        self.world_size, self.rank = geometry.world_size, geometry.rank
        self._name = f"sparknet-{uuid.uuid4().hex[:12]}-r{self.rank}"
        self._own = shared_memory.SharedMemory(name=self._name, create=True, size=geometry.region_bytes)
        self._peers: list[Optional[shared_memory.SharedMemory]] = [None] * self.world_size
        self._error = ""

    def local_blob(self) -> bytes:
        return json.dumps({"name": self._name, "bytes": self.geometry.region_bytes}).encode()

    def connect(self, group) -> None:
        import torch.distributed as dist

        blobs: list = [None] * self.world_size
        dist.all_gather_object(blobs, self.local_blob(), group=group)
        infos = [json.loads(b) for b in blobs]
        if len({i["bytes"] for i in infos}) != 1:
            self._error = "region sizes differ across ranks"
            raise RuntimeError(self._error)
        for peer, info in enumerate(infos):
            self._peers[peer] = self._own if peer == self.rank else shared_memory.SharedMemory(name=info["name"])
        dist.barrier(group=group)

    def start(self) -> None:
        return None

    def stop(self) -> None:
        return None

    def buffer(self, peer: int) -> memoryview:
        """The mapped region of ``peer`` (this rank's own for ``peer == rank``)."""
        shm = self._peers[peer]
        if shm is None:
            raise RuntimeError("transport is not connected")
        return shm.buf

    def bases(self) -> list[int]:
        import ctypes

        out = []
        for shm in self._peers:
            if shm is None:
                raise RuntimeError("transport is not connected")
            out.append(ctypes.addressof(ctypes.c_char.from_buffer(shm.buf)))
        return out

    def multicast(self) -> Optional[tuple[int, int, int]]:
        return None

    def failed(self) -> bool:
        return bool(self._error)

    def error(self) -> str:
        return self._error

    def stats(self) -> dict[str, Any]:
        return {"transport": self.name, "segment": self._name, "region_bytes": self.geometry.region_bytes}

    def close(self) -> None:
        for peer, shm in enumerate(self._peers):
            if shm is not None and peer != self.rank:
                shm.close()
        self._peers = [None] * self.world_size
        try:
            self._own.close()
            self._own.unlink()
        except FileNotFoundError:
            pass


__all__ = ["HostStagedTransport", "host_staged_capability"]
