"""Discover the local GPU map through NVML (replaces the reference's LLDP-over-ssh
cable discovery, ``sparknet/topology/discover.py:59-284``).

``local_inventory`` reads, for every GPU: index, name, UUID, PCI bus ID, NUMA node,
active NVLink count and each link's remote PCI device (an NVSwitch shows up as a
non-GPU remote), the NVLink P2P capability to every other GPU, and, through an
optional CUDA query, multicast (NVLS) support.  ``generate_map`` turns an inventory
into a validated map.  Everything goes through an ``nvml`` object with pynvml's
interface, so tests pass a fake and nothing here needs a GPU.  Read-only: no NVML
setter is called.
"""

from __future__ import annotations

import socket
from typing import Any, Callable, Optional

from . import gpumap


def _load_nvml():
    import pynvml  # nvidia-ml-py

    pynvml.nvmlInit()
    return pynvml


def _text(value) -> str:
    return value.decode() if isinstance(value, bytes) else str(value)


def _numa_node(nvml, handle) -> Optional[int]:
    getter = getattr(nvml, "nvmlDeviceGetNumaNodeId", None)
    if getter is None:
        return None
    try:
        return int(getter(handle))
    except Exception:  # noqa: BLE001 - not all drivers expose it
        return None


def _nvlinks(nvml, handle) -> tuple[int, list[str]]:
    active, remotes = 0, []
    for link in range(int(getattr(nvml, "NVML_NVLINK_MAX_LINKS", 18))):
        try:
            state = nvml.nvmlDeviceGetNvLinkState(handle, link)
        except Exception:  # noqa: BLE001 - link absent
            break
        if state == getattr(nvml, "NVML_FEATURE_ENABLED", 1):
            active += 1
            try:
                info = nvml.nvmlDeviceGetNvLinkRemotePciInfo_v2(handle, link)
                remotes.append(gpumap.normalize_pci(_text(info.busId)))
            except Exception:  # noqa: BLE001
                pass
    return active, remotes


def _p2p(nvml, a, b) -> bool:
    index = getattr(nvml, "NVML_P2P_CAPS_INDEX_NVLINK", 3)
    ok = getattr(nvml, "NVML_P2P_STATUS_OK", 0)
    try:
        return nvml.nvmlDeviceGetP2PStatus(a, b, index) == ok
    except Exception:  # noqa: BLE001
        return False


def cuda_multicast_query(index: int) -> bool:
    """CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED for device ``index`` (cuda-python)."""
    from cuda.bindings import driver

    driver.cuInit(0)
    err, dev = driver.cuDeviceGet(index)
    if err != driver.CUresult.CUDA_SUCCESS:
        return False
    err, value = driver.cuDeviceGetAttribute(driver.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev)
    return err == driver.CUresult.CUDA_SUCCESS and bool(value)


def local_inventory(nvml: Any = None, *, multicast: Optional[Callable[[int], bool]] = None) -> dict:
    """Every local GPU as NVML sees it, plus driver/CUDA versions."""
    nvml = nvml if nvml is not None else _load_nvml()
    count = int(nvml.nvmlDeviceGetCount())
    handles = [nvml.nvmlDeviceGetHandleByIndex(i) for i in range(count)]
    gpus = []
    pcis = []
    for i, h in enumerate(handles):
        pci = gpumap.normalize_pci(_text(nvml.nvmlDeviceGetPciInfo(h).busId))
        pcis.append(pci)
        links, remotes = _nvlinks(nvml, h)
        gpus.append({
            "index": i,
            "name": _text(nvml.nvmlDeviceGetName(h)),
            "uuid": _text(nvml.nvmlDeviceGetUUID(h)),
            "pci_bus_id": pci,
            "numa_node": _numa_node(nvml, h),
            "nvlinks_active": links,
            "nvlink_remotes": remotes,
            "p2p_peers": [j for j in range(count) if j != i and _p2p(nvml, h, handles[j])],
            "multicast": bool(multicast(i)) if multicast is not None else None,
        })
    gpu_pcis = set(pcis)
    nvswitch = bool(gpus) and all(g["nvlinks_active"] > 0 for g in gpus) and all(
        any(r not in gpu_pcis for r in g["nvlink_remotes"]) or not g["nvlink_remotes"] for g in gpus)
    try:
        driver = _text(nvml.nvmlSystemGetDriverVersion())
    except Exception:  # noqa: BLE001
        driver = None
    try:
        cuda = int(nvml.nvmlSystemGetCudaDriverVersion())
        cuda = f"{cuda // 1000}.{(cuda % 1000) // 10}"
    except Exception:  # noqa: BLE001
        cuda = None
    return {"host": socket.gethostname(), "driver": driver, "cuda": cuda, "nvswitch": nvswitch, "gpus": gpus}


def generate_map(inventory: dict, *, name: Optional[str] = None, management_ip: Optional[str] = None,
                 management_interface: Optional[str] = None, ranks: Optional[list[int]] = None) -> dict:
    """A one-node map from an inventory; ``ranks`` picks GPU indices in rank order (default: all)."""
    order = ranks if ranks is not None else [g["index"] for g in inventory["gpus"]]
    rank_of = {index: r for r, index in enumerate(order)}
    gpus = []
    for g in inventory["gpus"]:
        entry = {k: g[k] for k in ("index", "name", "uuid", "pci_bus_id", "numa_node", "nvlinks_active",
                                   "p2p_peers")}
        entry["multicast"] = bool(g.get("multicast"))
        entry["rank"] = rank_of.get(g["index"])
        gpus.append(entry)
    node = {"name": name or inventory.get("host") or "box", "head": True, "nvswitch": bool(inventory.get("nvswitch")),
            "gpus": gpus}
    if management_ip:
        node["management_ip"] = management_ip
    if management_interface:
        node["management_interface"] = management_interface
    if inventory.get("driver"):
        node["driver"] = inventory["driver"]
    if inventory.get("cuda"):
        node["cuda"] = inventory["cuda"]
    return {"schema_version": gpumap.SCHEMA_VERSION, "nodes": [node]}


__all__ = ["cuda_multicast_query", "generate_map", "local_inventory"]
