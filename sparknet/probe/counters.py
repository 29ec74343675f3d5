"""NVLink counters around a measurement (replaces the reference's RDMA and ethtool
counters, ``sparknet/probe/counters.py:17-56``).

``nvlink_counters`` reads, per GPU, the NVLink data throughput counters (bytes sent
and received, NVML field values) and the per-link error counters (CRC, replay,
recovery).  ``deltas`` subtracts two snapshots.  Read-only.
"""

from __future__ import annotations

from typing import Any

from . import nvml as nvml_mod

# NVML field ids (nvml.h): NVLink throughput, data only, summed over links.
FI_NVLINK_THROUGHPUT_DATA_TX = 138
FI_NVLINK_THROUGHPUT_DATA_RX = 139
ERROR_COUNTERS = {
    "replay": 0,      # NVML_NVLINK_ERROR_DL_REPLAY
    "recovery": 1,    # NVML_NVLINK_ERROR_DL_RECOVERY
    "crc_flit": 2,    # NVML_NVLINK_ERROR_DL_CRC_FLIT
    "crc_data": 3,    # NVML_NVLINK_ERROR_DL_CRC_DATA
}


def _field_values(nv, handle, ids):
    getter = getattr(nv, "nvmlDeviceGetFieldValues", None)
    if getter is None:
        return {}
    try:
        values = getter(handle, list(ids))
    except Exception:  # noqa: BLE001
        return {}
    out = {}
    for fid, v in zip(ids, values):
        if getattr(v, "nvmlReturn", 0) == 0:
            raw = getattr(v, "value", None)
            out[fid] = int(getattr(raw, "ullVal", raw if isinstance(raw, int) else 0))
    return out


def nvlink_counters(nvml: Any = None, *, links: int = 18) -> dict[str, int]:
    """Flat ``gpu<i>.<counter>`` -> value snapshot for every GPU."""
    nv = nvml if nvml is not None else nvml_mod.load()
    snap: dict[str, int] = {}
    for i, h in enumerate(nvml_mod.handles(nv)):
        fv = _field_values(nv, h, (FI_NVLINK_THROUGHPUT_DATA_TX, FI_NVLINK_THROUGHPUT_DATA_RX))
        if FI_NVLINK_THROUGHPUT_DATA_TX in fv:
            snap[f"gpu{i}.nvlink_tx_kib"] = fv[FI_NVLINK_THROUGHPUT_DATA_TX]
        if FI_NVLINK_THROUGHPUT_DATA_RX in fv:
            snap[f"gpu{i}.nvlink_rx_kib"] = fv[FI_NVLINK_THROUGHPUT_DATA_RX]
        for name, code in ERROR_COUNTERS.items():
            total = 0
            for link in range(links):
                try:
                    total += int(nv.nvmlDeviceGetNvLinkErrorCounter(h, link, code))
                except Exception:  # noqa: BLE001
                    break
            snap[f"gpu{i}.nvlink_{name}"] = total
    return snap


def own_gpu_counters(device_index: int, nvml: Any = None) -> dict[str, int]:
    """NVLink data counters (KiB sent and received) of the GPU behind the CUDA device
    ``device_index`` of this process, found by PCI bus id so that other jobs' GPUs on a
    shared box are never read.  Empty when NVML or the field is unavailable."""
    try:
        import torch

        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        nv = nvml if nvml is not None else nvml_mod.load()
        handle = nv.nvmlDeviceGetHandleByPciBusId_v2(bus)
    except Exception:  # noqa: BLE001 - counters are evidence, never a reason to fail a probe
        return {}
    fv = _field_values(nv, handle, (FI_NVLINK_THROUGHPUT_DATA_TX, FI_NVLINK_THROUGHPUT_DATA_RX))
    out = {}
    if FI_NVLINK_THROUGHPUT_DATA_TX in fv:
        out["nvlink_tx_kib"] = fv[FI_NVLINK_THROUGHPUT_DATA_TX]
    if FI_NVLINK_THROUGHPUT_DATA_RX in fv:
        out["nvlink_rx_kib"] = fv[FI_NVLINK_THROUGHPUT_DATA_RX]
    return out


def deltas(before: dict[str, int], after: dict[str, int]) -> dict[str, int]:
    """The counters that changed between two snapshots, as after minus before."""
    return {k: after[k] - before[k] for k in after if k in before and after[k] != before[k]}


def error_deltas(before: dict[str, int], after: dict[str, int]) -> dict[str, int]:
    """Only the error counters that moved (throughput is expected to move)."""
    return {k: v for k, v in deltas(before, after).items() if "nvlink_tx" not in k and "nvlink_rx" not in k}


__all__ = ["ERROR_COUNTERS", "deltas", "error_deltas", "nvlink_counters", "own_gpu_counters"]
