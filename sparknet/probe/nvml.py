"""Thin access to NVML (nvidia-ml-py) with a seam for tests.

Every probe module takes an ``nvml`` argument with pynvml's interface; ``load()``
returns the real module (initialised) or raises a clear error on a host without a
driver.  Nothing in the probe calls an NVML setter.
"""

from __future__ import annotations


def load():
    try:
        import pynvml
    except ImportError as exc:  # pragma: no cover - nvidia-ml-py is in the image
        raise RuntimeError("nvidia-ml-py (pynvml) is not installed") from exc
    try:
        pynvml.nvmlInit()
    except Exception as exc:  # noqa: BLE001
        raise RuntimeError(f"NVML is not available on this host: {exc}") from exc
    return pynvml


def text(value) -> str:
    return value.decode() if isinstance(value, bytes) else str(value)


def handles(nvml) -> list:
    return [nvml.nvmlDeviceGetHandleByIndex(i) for i in range(int(nvml.nvmlDeviceGetCount()))]
