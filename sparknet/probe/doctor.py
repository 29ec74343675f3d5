"""Read-only checks of one box against its GPU map before any process starts
(replaces the reference's RDMA doctor, ``sparknet/probe/doctor.py:13-71``).

Checks: the map validates for the transport; every mapped GPU is present (by UUID
and PCI bus ID); every tensor-parallel GPU has its NVLinks up; peers are P2P-capable
over NVLink; persistence mode is on and compute mode is Default (so several ranks
may open the device); ECC reports no volatile uncorrectable errors; no foreign
process already holds a tensor-parallel GPU; the driver matches the map; the
nvidia-fabricmanager service is running (NVSwitch boxes need it for NVLink P2P and
NVLS); and the build tools the runtime needs are present.  It reads only.
"""

from __future__ import annotations

import shutil
import subprocess
from typing import Any, Callable, Optional

from sparknet.topology import gpumap

from . import nvml as nvml_mod


def fabricmanager_active(run: Callable[..., Any] = subprocess.run) -> Optional[bool]:
    """True/False from systemd, None when systemd cannot say (containers)."""
    if shutil.which("systemctl") is None:
        return None
    try:
        out = run(["systemctl", "is-active", "nvidia-fabricmanager"], capture_output=True, text=True, timeout=5)
    except Exception:  # noqa: BLE001
        return None
    state = (out.stdout or "").strip()
    return state == "active" if state else None


def local_problems(gmap: dict, node_name: str, transport: str, *, nvml: Any = None,
                   fabricmanager: Optional[Callable[[], Optional[bool]]] = None,
                   which: Callable[[str], Optional[str]] = shutil.which) -> list[str]:
    """What keeps this host from serving ``node_name`` of the map over ``transport`` (read-
    only NVML checks; empty when ready)."""
    errors = gpumap.problems(gmap, transport)
    if errors:
        return errors
    node = gpumap.node_by_name(gmap, node_name)
    try:
        nv = nvml if nvml is not None else nvml_mod.load()
    except RuntimeError as exc:
        return [str(exc)]
    present = {}
    for h in nvml_mod.handles(nv):
        present[nvml_mod.text(nv.nvmlDeviceGetUUID(h))] = h
    ranked = gpumap.ranked_gpus(node)
    index_of = {}
    for g in ranked:
        h = present.get(g["uuid"])
        label = f"rank {g['rank']} ({g['uuid']})"
        if h is None:
            errors.append(f"{label}: GPU not present on this host")
            continue
        index_of[g["index"]] = h
        pci = gpumap.normalize_pci(nvml_mod.text(nv.nvmlDeviceGetPciInfo(h).busId))
        if pci != gpumap.normalize_pci(g["pci_bus_id"]):
            errors.append(f"{label}: PCI bus ID is {pci}, the map says {g['pci_bus_id']}")
        active = 0
        for link in range(int(getattr(nv, "NVML_NVLINK_MAX_LINKS", 18))):
            try:
                if nv.nvmlDeviceGetNvLinkState(h, link) == getattr(nv, "NVML_FEATURE_ENABLED", 1):
                    active += 1
            except Exception:  # noqa: BLE001
                break
        if active < int(g.get("nvlinks_active", 0)):
            errors.append(f"{label}: {active} NVLinks active, the map expects {g['nvlinks_active']}")
        try:
            if nv.nvmlDeviceGetPersistenceMode(h) != getattr(nv, "NVML_FEATURE_ENABLED", 1):
                errors.append(f"{label}: persistence mode is off (first CUDA init per process pays the driver "
                              "load; an operator enables it, this probe does not)")
        except Exception:  # noqa: BLE001
            pass
        try:
            if nv.nvmlDeviceGetComputeMode(h) != getattr(nv, "NVML_COMPUTEMODE_DEFAULT", 0):
                errors.append(f"{label}: compute mode is not Default")
        except Exception:  # noqa: BLE001
            pass
        try:
            ecc = nv.nvmlDeviceGetTotalEccErrors(h, getattr(nv, "NVML_MEMORY_ERROR_TYPE_UNCORRECTED", 1),
                                                 getattr(nv, "NVML_VOLATILE_ECC", 0))
            if int(ecc) > 0:
                errors.append(f"{label}: {int(ecc)} volatile uncorrectable ECC errors")
        except Exception:  # noqa: BLE001
            pass
        try:
            procs = nv.nvmlDeviceGetComputeRunningProcesses(h)
            if procs:
                errors.append(f"{label}: {len(procs)} process(es) already hold this GPU")
        except Exception:  # noqa: BLE001
            pass
    if gpumap.uses_oneshot(transport) and len(ranked) > 1:
        p2p = getattr(nv, "NVML_P2P_CAPS_INDEX_NVLINK", 3)
        ok = getattr(nv, "NVML_P2P_STATUS_OK", 0)
        for a_index, a in index_of.items():
            for b_index, b in index_of.items():
                if a_index < b_index:
                    try:
                        status = nv.nvmlDeviceGetP2PStatus(a, b, p2p)
                    except Exception:  # noqa: BLE001
                        status = None
                    if status != ok:
                        errors.append(f"GPUs {a_index} and {b_index}: no NVLink peer-to-peer path")
    expected_driver = node.get("driver")
    if expected_driver:
        try:
            driver = nvml_mod.text(nv.nvmlSystemGetDriverVersion())
            if driver != expected_driver:
                errors.append(f"driver {driver} differs from the map's {expected_driver}")
        except Exception:  # noqa: BLE001
            pass
    if node.get("nvswitch") and len(ranked) > 1:
        state = (fabricmanager or fabricmanager_active)()
        if state is False:
            errors.append("nvidia-fabricmanager is not active: NVSwitch peer traffic and NVLS need it")
    if which("nvcc") is None:
        errors.append("nvcc not found: the sm_100a extension cannot be rebuilt on this host")
    return errors


__all__ = ["fabricmanager_active", "local_problems"]
