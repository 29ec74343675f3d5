"""What this host offers the NVLink transport (replaces the reference's GPUDirect
readiness report, ``sparknet/probe/gpudirect.py:37-90``).

Reports: driver and CUDA versions, GPU count and names, the NVLink P2P matrix, active
link counts, NVSwitch presence, multicast (NVLS) support, fabric handle support (the
handle type multi-node NVLink needs; single boxes use POSIX descriptors), IMEX
channel devices, and the fabric manager state; then a readiness verdict per stage:
``p2p`` (one-shot/two-shot kernels), ``nvls`` (multimem kernels), ``fabric``
(cross-box NVLink).  Read-only.
"""

from __future__ import annotations

import os
from typing import Any, Callable, Optional

from . import nvml as nvml_mod
from .doctor import fabricmanager_active

CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED = 132
CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_FABRIC_SUPPORTED = 128


def _cuda_attr(index: int, attr: int) -> Optional[int]:
    try:
        from cuda.bindings import driver
    except ImportError:
        return None
    try:
        driver.cuInit(0)
        err, dev = driver.cuDeviceGet(index)
        if err != driver.CUresult.CUDA_SUCCESS:
            return None
        err, value = driver.cuDeviceGetAttribute(driver.CUdevice_attribute(attr), dev)
        return int(value) if err == driver.CUresult.CUDA_SUCCESS else None
    except Exception:  # noqa: BLE001
        return None


def nvlink_report(*, nvml: Any = None, cuda_attr: Callable[[int, int], Optional[int]] = _cuda_attr,
                  fabricmanager: Callable[[], Optional[bool]] = fabricmanager_active, dev_root: str = "/dev") -> dict:
    """What this host offers the NVLink transport: P2P pairs, multicast, fabric handles,
    IMEX channels and the fabric manager, with a readiness verdict per stage."""
    try:
        nv = nvml if nvml is not None else nvml_mod.load()
    except RuntimeError as exc:
        return {"error": str(exc), "ready": {"p2p": False, "nvls": False, "fabric": False}}
    hs = nvml_mod.handles(nv)
    gpus, matrix = [], []
    p2p = getattr(nv, "NVML_P2P_CAPS_INDEX_NVLINK", 3)
    ok = getattr(nv, "NVML_P2P_STATUS_OK", 0)
    for i, h in enumerate(hs):
        links = 0
        for link in range(int(getattr(nv, "NVML_NVLINK_MAX_LINKS", 18))):
            try:
                if nv.nvmlDeviceGetNvLinkState(h, link) == getattr(nv, "NVML_FEATURE_ENABLED", 1):
                    links += 1
            except Exception:  # noqa: BLE001
                break
        gpus.append({"index": i, "name": nvml_mod.text(nv.nvmlDeviceGetName(h)), "nvlinks_active": links,
                     "multicast": cuda_attr(i, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED),
                     "fabric_handles": cuda_attr(i, CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_FABRIC_SUPPORTED)})
        row = []
        for j, g in enumerate(hs):
            if i == j:
                row.append("X")
                continue
            try:
                row.append("OK" if nv.nvmlDeviceGetP2PStatus(h, g, p2p) == ok else "NO")
            except Exception:  # noqa: BLE001
                row.append("?")
        matrix.append(row)
    imex = sorted(os.listdir(os.path.join(dev_root, "nvidia-caps-imex-channels"))) \
        if os.path.isdir(os.path.join(dev_root, "nvidia-caps-imex-channels")) else []
    try:
        driver = nvml_mod.text(nv.nvmlSystemGetDriverVersion())
    except Exception:  # noqa: BLE001
        driver = None
    all_p2p = all(cell in ("X", "OK") for row in matrix for cell in row)
    fm = fabricmanager()
    ready = {
        "p2p": bool(gpus) and all_p2p and all(g["nvlinks_active"] > 0 for g in gpus) and fm is not False,
        "nvls": bool(gpus) and all(g["multicast"] for g in gpus) and fm is not False,
        "fabric": bool(gpus) and all(g["fabric_handles"] for g in gpus) and bool(imex),
    }
    return {"driver": driver, "gpus": gpus, "p2p_matrix": matrix, "imex_channels": imex,
            "fabricmanager_active": fm, "ready": ready}


def render(report: dict) -> str:
    """The report as text."""
    if "error" in report:
        return f"NVLink report unavailable: {report['error']}\n"
    lines = [f"driver {report['driver']}, {len(report['gpus'])} GPU(s), fabric manager "
             f"{ {True: 'active', False: 'inactive', None: 'unknown'}[report['fabricmanager_active']] }"]
    for g in report["gpus"]:
        lines.append(f"  gpu{g['index']} {g['name']}: {g['nvlinks_active']} NVLinks, multicast={g['multicast']}, "
                     f"fabric handles={g['fabric_handles']}")
    lines.append("  P2P over NVLink:")
    for i, row in enumerate(report["p2p_matrix"]):
        lines.append(f"    gpu{i}: " + " ".join(f"{c:>2}" for c in row))
    for stage, ready in report["ready"].items():
        lines.append(f"  {stage}: {'ready' if ready else 'not ready'}")
    return "\n".join(lines) + "\n"


__all__ = ["nvlink_report", "render"]
