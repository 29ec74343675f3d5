"""Read-only fabric checks and the model-free collective probe for NVSwitch boxes.

- ``doctor``: the GPU map against this host (NVML), before any process starts.
- ``counters``: NVLink throughput and error counters around a measurement.
- ``nvlink_report``: what the host offers the transport (P2P, NVLS, fabric handles).
- ``container``: the bounded container command that runs the probe on one box.
- ``fleet``: runs that command on every box of a map and keeps the receipts.
- ``summary``: latency tables from the receipts.
- ``collectives``: the torch.distributed probe (needs torch; one rank per GPU).
- ``failstop``: fail-stop qualification without faulting a GPU.
"""

from .container import docker_probe_command
from .counters import deltas, nvlink_counters
from .doctor import local_problems
from .nvlink_report import nvlink_report

# The reference's host capability report (GPUDirect RDMA readiness) is, on an NVSwitch
# box, the NVLink report: the same question (what does this host offer the
# collectives' transport) for the transport used here.  `sparknet probe gpudirect`
# prints it too.
gpudirect_report = nvlink_report

__all__ = ["deltas", "docker_probe_command", "gpudirect_report", "local_problems", "nvlink_counters",
           "nvlink_report"]
