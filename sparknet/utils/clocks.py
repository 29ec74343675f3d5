"""Sample GPU clocks and throttle reasons while a measurement runs.

``ClockSampler`` starts ``nvidia-smi --query-gpu ... -lms <interval>`` in the
background and, when stopped, summarises the samples taken under load: median SM
clock, the maximum clock and the throttle reasons seen.  Start it before the warm-up
(nvidia-smi needs a moment to begin) and bracket the timed region with
``mark_start()`` / ``mark_end()``: only samples stamped inside that window count, or,
for a window shorter than the sampling interval, the samples nearest to it.  It only
reads settings; it never changes a clock, power limit or any other GPU state.
"""

from __future__ import annotations

import atexit
import csv
import io
import os
import shutil
import statistics
import subprocess
import tempfile
import time
from datetime import datetime

FIELDS = ("index", "clocks.sm", "clocks.max.sm", "power.draw", "utilization.gpu",
          "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
          "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap", "timestamp")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
REJECTING = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def _num(text: str) -> float | None:
    text = text.strip().split(" ")[0]
    try:
        return float(text)
    except ValueError:
        return None


def _stamp(text: str) -> float | None:
    """nvidia-smi's ``timestamp`` field (local time) as epoch seconds."""
    try:
        return datetime.strptime(text.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
    except ValueError:
        return None


def summarize(csv_text: str, gpus: list[int] | None = None, window: tuple[float, float] | None = None,
              slack_s: float = 0.25) -> dict:
    """Median SM clock over samples with the GPU busy, max clock, and active reasons.

    ``window`` (epoch seconds) keeps the samples stamped inside it; if none are, the
    ones within ``slack_s`` of it (a window shorter than the sampling interval)."""
    rows = [r for r in csv.reader(io.StringIO(csv_text)) if len(r) >= 9 and r[0].strip().isdigit()]
    if gpus is not None:
        rows = [r for r in rows if int(r[0]) in gpus]
    in_window = None
    loaded = False  # rows stamped inside the timed window are under load by construction
    if window is not None:
        t0, t1 = window
        stamped = [(r, _stamp(r[9]) if len(r) > 9 else None) for r in rows]
        inside = [r for r, t in stamped if t is not None and t0 <= t <= t1]
        near = [r for r, t in stamped if t is not None and t0 - slack_s <= t <= t1 + slack_s]
        in_window = len(inside)
        rows = inside or near
        loaded = bool(inside)
    mhz, busy_mhz, max_mhz, reasons = [], [], None, set()
    for row in rows:
        sm, smax, util = _num(row[1]), _num(row[2]), _num(row[4])
        if sm is None:
            continue
        mhz.append(sm)
        # NVML's utilisation averages over longer than a short window: inside the
        # window a sample counts as loaded whatever it says
        if loaded or (util is not None and util > 0):
            busy_mhz.append(sm)
        if smax is not None:
            max_mhz = smax if max_mhz is None else max(max_mhz, smax)
        for name, value in zip(REASONS, row[5:9]):
            if value.strip().lower() == "active":
                reasons.add(name)
    # only samples with the GPU busy speak for the clock under load (an idle GPU parks
    # its clock low); without any, report none rather than an idle clock
    out = {
        "sm_mhz": statistics.median(busy_mhz) if busy_mhz else None,
        "sm_mhz_any": statistics.median(mhz) if mhz else None,
        "sm_max_mhz": max_mhz,
        "reasons": sorted(reasons),
        "samples": len(mhz),
        "samples_under_load": len(busy_mhz),
        "rejected": bool(reasons & set(REJECTING)),
    }
    if in_window is not None:
        out["samples_in_window"] = in_window
    return out


class ClockSampler:
    def __init__(self, gpus: list[int] | None = None, interval_ms: int = 200):
        self.gpus = gpus
        self.interval_ms = interval_ms
        self._proc = None
        self._file = None
        self._t0 = None
        self._t1 = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        self._file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = [exe, f"--query-gpu={','.join(FIELDS)}", "--format=csv,noheader", f"-lms={self.interval_ms}"]
        if self.gpus is not None:
            cmd.append("--id=" + ",".join(str(g) for g in self.gpus))
        self._proc = subprocess.Popen(cmd, stdout=self._file, stderr=subprocess.DEVNULL)
        atexit.register(self._abandon)  # a run that fails before stop() must not leave the sampler running
        return self

    def _abandon(self) -> None:
        """Stop this sampler's own process (exactly that PID) and drop its file."""
        proc, self._proc = self._proc, None
        if proc is not None and proc.poll() is None:
            proc.terminate()
            try:
                proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                proc.kill()
        if self._file is not None:
            try:
                self._file.close()
                os.unlink(self._file.name)
            except OSError:
                pass

    def mark_start(self) -> None:
        self._t0 = time.time()

    def mark_end(self) -> None:
        self._t1 = time.time()

    def stop(self) -> dict:
        if self._proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi absent"}
        if self._t0 is not None and self._t1 is None:
            self.mark_end()
        time.sleep(min(1.0, 2 * self.interval_ms / 1000.0))  # let the sample after the window land
        atexit.unregister(self._abandon)
        self._proc.terminate()
        try:
            self._proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self._proc.kill()
            self._proc.wait()
        self._proc = None
        self._file.flush()
        self._file.seek(0)
        text = self._file.read()
        self._file.close()
        os.unlink(self._file.name)
        window = (self._t0, self._t1) if self._t0 is not None else None
        return summarize(text, None, window=window)
