"""Sample GPU clocks and throttle reasons while a measurement runs.

``ClockSampler`` starts ``nvidia-smi --query-gpu ... -lms 200`` in the background
and, when stopped, summarises the samples taken under load: median SM clock, the
maximum clock and the throttle reasons seen.  It only reads settings; it never
changes a clock, power limit or any other GPU state.
"""

from __future__ import annotations

import csv
import io
import os
import shutil
import statistics
import subprocess
import tempfile

FIELDS = ("index", "clocks.sm", "clocks.max.sm", "power.draw", "utilization.gpu",
          "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
          "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
REJECTING = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def _num(text: str) -> float | None:
    text = text.strip().split(" ")[0]
    try:
        return float(text)
    except ValueError:
        return None


def summarize(csv_text: str, gpus: list[int] | None = None) -> dict:
    """Median SM clock over samples with the GPU busy, max clock, and active reasons."""
    rows = list(csv.reader(io.StringIO(csv_text)))
    mhz, busy_mhz, max_mhz, reasons = [], [], None, set()
    for row in rows:
        if len(row) < len(FIELDS) or not row[0].strip().isdigit():
            continue
        index = int(row[0])
        if gpus is not None and index not in gpus:
            continue
        sm, smax, util = _num(row[1]), _num(row[2]), _num(row[4])
        if sm is None:
            continue
        mhz.append(sm)
        if util is not None and util > 0:
            busy_mhz.append(sm)
        if smax is not None:
            max_mhz = smax if max_mhz is None else max(max_mhz, smax)
        for name, value in zip(REASONS, row[5:9]):
            if value.strip().lower() == "active":
                reasons.add(name)
    use = busy_mhz or mhz
    return {
        "sm_mhz": statistics.median(use) if use else None,
        "sm_max_mhz": max_mhz,
        "reasons": sorted(reasons),
        "samples": len(mhz),
        "samples_under_load": len(busy_mhz),
        "rejected": bool(reasons & set(REJECTING)),
    }


class ClockSampler:
    def __init__(self, gpus: list[int] | None = None, interval_ms: int = 200):
        self.gpus = gpus
        self.interval_ms = interval_ms
        self._proc = None
        self._file = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        self._file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = [exe, f"--query-gpu={','.join(FIELDS)}", "--format=csv,noheader", f"-lms={self.interval_ms}"]
        if self.gpus is not None:
            cmd.append("--id=" + ",".join(str(g) for g in self.gpus))
        self._proc = subprocess.Popen(cmd, stdout=self._file, stderr=subprocess.DEVNULL)
        return self

    def stop(self) -> dict:
        if self._proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi absent"}
        self._proc.terminate()
        try:
            self._proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self._proc.kill()
            self._proc.wait()
        self._file.flush()
        self._file.seek(0)
        text = self._file.read()
        self._file.close()
        os.unlink(self._file.name)
        return summarize(text, None)
