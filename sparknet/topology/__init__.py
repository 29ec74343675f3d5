"""GPU maps for NVSwitch boxes: schema, validation, subsets, environment rendering, NVML discovery.

CPU-only; imports nothing from torch.
"""

from .gpumap import (
    ONESHOT_TRANSPORTS,
    SCHEMA_VERSION,
    TRANSPORTS,
    WORLD_SIZES,
    gpu_by_rank,
    head_node,
    load,
    node_by_name,
    normalize_pci,
    problems,
    ranked_gpus,
    subset,
    uses_nvls,
    uses_oneshot,
    world_size,
)
from .render import OWNED_KEYS, base_problems, environment_problems, node_environment, visible_devices

__all__ = [
    "ONESHOT_TRANSPORTS", "OWNED_KEYS", "SCHEMA_VERSION", "TRANSPORTS", "WORLD_SIZES", "base_problems",
    "environment_problems", "gpu_by_rank", "head_node", "load", "node_by_name", "node_environment", "normalize_pci",
    "problems", "ranked_gpus", "subset", "uses_nvls", "uses_oneshot", "visible_devices", "world_size",
]
