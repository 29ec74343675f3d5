"""NVLink transports: peer-to-peer symmetric regions, optionally with NVLS multicast.

``NvlinkP2PTransport`` wraps the native bootstrap (``csrc/symm_mem.cpp``): a VMM
region per rank, descriptors passed over abstract unix sockets, peers mapped
read/write.  ``NvlsTransport`` adds the multicast object.  Both are device-initiated:
``start``/``stop`` have nothing to run (there is no proxy thread).
"""

from __future__ import annotations

import json
import os
import shutil
from typing import Any, Optional

from .base import Geometry, TransportCapability


def nvlink_capability(device_index: int = 0) -> TransportCapability:
    """Whether this host can run the NVLink transport on ``device_index`` (and why not)."""
    reasons, details = [], {}
    try:
        from sparknet import _native

        C = _native.load()
        details["vmm_granularity"] = int(C.vmm_granularity(device_index))
        details["multicast"] = bool(C.multicast_supported(device_index))
    except Exception as exc:  # noqa: BLE001 - reported as a reason
        reasons.append(str(exc))
    if shutil.which("nvidia-smi") is None:
        reasons.append("nvidia-smi not found (no driver?)")
    return TransportCapability(name="nvlink-p2p", available=not reasons, reasons=tuple(reasons), details=details)


class NvlinkP2PTransport:
    """Symmetric regions over NVLink: a CUDA VMM region per rank, descriptors passed to the
    peers, every peer's region mapped."""
    name = "nvlink-p2p"

    def __init__(self, geometry: Geometry):
        problems = geometry.validate()
        if problems:
            raise ValueError("; ".join(problems))
        self.geometry = geometry
        self.world_size, self.rank = geometry.world_size, geometry.rank
        self._regions = None
        self._error = ""
        self._connected = False

    def _multicast_bytes(self) -> int:
        return 0

    def local_blob(self) -> bytes:
        return json.dumps({"pid": os.getpid(), "rank": self.rank, "region_bytes": self.geometry.region_bytes,
                           "device": self.geometry.device_index}).encode()

    def connect(self, group) -> None:
        from sparknet import _native
        from sparknet.oneshot import symm

        try:
            self._regions = symm.build_regions(_native.load(), group=group, device_index=self.geometry.device_index,
                                               region_bytes=self.geometry.region_bytes,
                                               multicast_bytes=self._multicast_bytes())
            self._connected = True
        except Exception as exc:
            self._error = str(exc)
            raise

    def start(self) -> None:
        return None

    def stop(self) -> None:
        return None

    def bases(self) -> list[int]:
        if self._regions is None:
            raise RuntimeError("transport is not connected")
        return list(self._regions.bases)

    def multicast(self) -> Optional[tuple[int, int, int]]:
        if self._regions is None or self._regions.multicast is None:
            return None
        return self._regions.mc_ptr, self._regions.mc_uc_ptr, self._regions.mc_bytes

    def failed(self) -> bool:
        return bool(self._error)

    def error(self) -> str:
        return self._error

    def stats(self) -> dict[str, Any]:
        return {"transport": self.name, "connected": self._connected, "region_bytes": self.geometry.region_bytes,
                "multicast": self.multicast() is not None}

    def close(self) -> None:
        self._regions = None
        self._connected = False


class NvlsTransport(NvlinkP2PTransport):
    """The NVLink transport plus an NVLS multicast object bound to every rank's buffer."""
    name = "nvlink-nvls"

    def _multicast_bytes(self) -> int:
        return self.geometry.multicast_bytes


__all__ = ["NvlinkP2PTransport", "NvlsTransport", "nvlink_capability"]
