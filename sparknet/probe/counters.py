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


# Blackwell's byte counters (per link: scope = link index), used where the
# throughput fields above are not offered.
FI_NVLINK_COUNT_XMIT_BYTES = 202
FI_NVLINK_COUNT_RCV_BYTES = 204


def _handle_of_device(nv, device_index: int):
    """The NVML handle of this process's CUDA device ``device_index``, matched by PCI bus
    id (so another job's GPU on a shared box is never read)."""
    import torch

    props = torch.cuda.get_device_properties(device_index)
    want = (int(props.pci_domain_id), int(props.pci_bus_id), int(props.pci_device_id))
    for h in nvml_mod.handles(nv):
        info = nv.nvmlDeviceGetPciInfo(h)
        if (int(info.domain), int(info.bus), int(info.device)) == want:
            return h
    raise LookupError(f"no NVML device at PCI {want}")


def _scoped_sum(nv, handle, field: int, links: int):
    getter = getattr(nv, "nvmlDeviceGetFieldValues", None)
    if getter is None:
        return None
    try:
        values = getter(handle, [(field, link) for link in range(links)])
    except Exception:  # noqa: BLE001
        return None
    total, seen = 0, 0
    for v in values:
        if getattr(v, "nvmlReturn", 1) == 0:
            raw = getattr(v, "value", None)
            total += int(getattr(raw, "ullVal", raw if isinstance(raw, int) else 0))
            seen += 1
    return total if seen else None


def own_gpu_counters(device_index: int, nvml: Any = None, *, links: int = 18) -> dict:
    """NVLink bytes sent and received so far by the GPU behind the CUDA device
    ``device_index`` of this process: ``nvlink_tx_bytes`` / ``nvlink_rx_bytes`` and the
    NVML source used.  Tries the aggregate data-throughput fields (KiB), then the
    per-link byte counters summed over links.  Empty (with ``why``) when NVML offers
    neither: counters are evidence, never a reason to fail a probe."""
    try:
        nv = nvml if nvml is not None else nvml_mod.load()
        handle = _handle_of_device(nv, device_index)
    except Exception as exc:  # noqa: BLE001
        return {"why": f"{type(exc).__name__}: {exc}"}
    fv = _field_values(nv, handle, (FI_NVLINK_THROUGHPUT_DATA_TX, FI_NVLINK_THROUGHPUT_DATA_RX))
    if FI_NVLINK_THROUGHPUT_DATA_TX in fv and FI_NVLINK_THROUGHPUT_DATA_RX in fv:
        return {"nvlink_tx_bytes": fv[FI_NVLINK_THROUGHPUT_DATA_TX] * 1024,
                "nvlink_rx_bytes": fv[FI_NVLINK_THROUGHPUT_DATA_RX] * 1024, "source": "throughput_data_kib"}
    tx = _scoped_sum(nv, handle, FI_NVLINK_COUNT_XMIT_BYTES, links)
    rx = _scoped_sum(nv, handle, FI_NVLINK_COUNT_RCV_BYTES, links)
    if tx is not None and rx is not None:
        return {"nvlink_tx_bytes": tx, "nvlink_rx_bytes": rx, "source": "count_bytes_per_link"}
    return {"why": "NVML offers neither NVLink throughput fields nor per-link byte counters here"}


def deltas(before: dict[str, int], after: dict[str, int]) -> dict[str, int]:
    """The counters that changed between two snapshots, as after minus before."""
    return {k: after[k] - before[k] for k in after if k in before and after[k] != before[k]}


def error_deltas(before: dict[str, int], after: dict[str, int]) -> dict[str, int]:
    """Only the error counters that moved (throughput is expected to move)."""
    return {k: v for k, v in deltas(before, after).items() if "nvlink_tx" not in k and "nvlink_rx" not in k}


__all__ = ["ERROR_COUNTERS", "deltas", "error_deltas", "nvlink_counters", "own_gpu_counters"]
