"""``sparknet.oneshot``: NVLink collectives for tensor-parallel inference on B200.

``AllReduce`` is the runtime (``from_exchange_group``, ``prepare``,
``should_allreduce``, ``all_reduce``, ``all_reduce_residual_rmsnorm``,
``should_all_gather``, ``all_gather``, ``should_reduce_scatter``,
``reduce_scatter``, ``should_exchange``, ``exchange``, ``should_all_to_all_rows``,
``all_to_all_rows``, ``capture``, ``check_health``, ``failure``,
``set_timeout_ms``, ``poisoned``, ``reset``, ``stats``, ``close``).

Importing this package imports torch.  The kernels are compiled ahead of time into
``sparknet._C`` (``python setup.py build_ext --inplace``).
"""

from __future__ import annotations

from ._freeze import (
    KernelResolutionFrozenError,
    freeze_kernel_resolution,
    kernel_resolution_frozen,
    thaw_kernel_resolution,
)
from .runtime import (
    API_VERSION,
    DEFAULT_MAX_GATHER_BYTES,
    DEFAULT_MAX_SIZE,
    SUPPORTED_DTYPES,
    SUPPORTED_WORLD_SIZES,
    TOPOLOGIES,
    NvlinkAllReduce,
    discover_hcas,
    discover_nvlink_gpus,
    is_supported,
)

AllReduce = NvlinkAllReduce

__all__ = [
    "API_VERSION", "AllReduce", "DEFAULT_MAX_GATHER_BYTES", "DEFAULT_MAX_SIZE", "KernelResolutionFrozenError",
    "NvlinkAllReduce", "SUPPORTED_DTYPES", "SUPPORTED_WORLD_SIZES", "TOPOLOGIES", "discover_hcas",
    "discover_nvlink_gpus", "freeze_kernel_resolution", "is_supported", "kernel_resolution_frozen",
    "thaw_kernel_resolution",
]
