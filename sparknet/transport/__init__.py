"""The transport seam of the NVLink collectives.

The GPU protocol (device epoch, parity slots, Lamport/LL arrival markers, fixed-rank
reduction) does not depend on how the symmetric regions were made.
``NvlinkP2PTransport`` (VMM regions mapped peer-to-peer) and ``NvlsTransport`` (plus
an NVLS multicast object) are the device transports; ``HostStagedTransport`` is a
host-memory double for CPU tests.
"""

from .base import Geometry, Transport, TransportCapability
from .host_staged import HostStagedTransport, host_staged_capability
from .nvlink import NvlinkP2PTransport, NvlsTransport, nvlink_capability

__all__ = ["Geometry", "HostStagedTransport", "NvlinkP2PTransport", "NvlsTransport", "Transport",
           "TransportCapability", "host_staged_capability", "nvlink_capability"]
