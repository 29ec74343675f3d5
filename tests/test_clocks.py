"""Clock-sample summaries (CPU): busy samples only, throttle reasons, the timed window."""

from datetime import datetime

from sparknet.utils import clocks


def _row(index, sm, util, reasons=("Not Active",) * 4, ts=None):
    stamp = ts.strftime("%Y/%m/%d %H:%M:%S.%f")[:-3] if ts else "2026/12/02 10:00:00.000"
    return ", ".join([str(index), f"{sm} MHz", "1965 MHz", "900.00 W", f"{util} %", *reasons, stamp])


def test_summary_uses_busy_samples_and_reasons():
    text = "\n".join([_row(0, 120, 0), _row(0, 1900, 95), _row(0, 1850, 97),
                      _row(0, 1300, 99, ("Not Active", "Not Active", "Not Active", "Active"))])
    s = clocks.summarize(text)
    assert s["sm_mhz"] == 1850 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"] and not s["rejected"]
    hot = clocks.summarize(_row(0, 1500, 90, ("Not Active", "Active", "Not Active", "Not Active")))
    assert hot["rejected"] and hot["reasons"] == ["hw_thermal_slowdown"]


def test_idle_only_reports_no_clock():
    s = clocks.summarize("\n".join([_row(0, 120, 0), _row(0, 345, 0)]))
    assert s["sm_mhz"] is None and s["sm_mhz_any"] == 232.5


def test_window_keeps_inside_or_nearest_samples():
    t = datetime(2026, 12, 2, 10, 0, 0, 500000)
    base = t.timestamp()
    rows = [_row(0, 1000, 50, ts=datetime.fromtimestamp(base - 2)),
            _row(0, 1900, 90, ts=datetime.fromtimestamp(base + 0.01)),
            _row(0, 1000, 50, ts=datetime.fromtimestamp(base + 3))]
    s = clocks.summarize("\n".join(rows), window=(base, base + 0.02))
    assert s["sm_mhz"] == 1900 and s["samples_in_window"] == 1 and s["samples"] == 1
    # a window between samples takes the ones within the slack
    s = clocks.summarize("\n".join(rows), window=(base + 0.05, base + 0.06), slack_s=0.1)
    assert s["samples_in_window"] == 0 and s["sm_mhz"] == 1900


def test_samples_inside_the_window_count_as_loaded():
    t = datetime(2026, 12, 2, 10, 0, 0, 500000)
    base = t.timestamp()
    rows = [_row(0, 1965, 0, ts=datetime.fromtimestamp(base + 0.01)),
            _row(0, 1965, 0, ts=datetime.fromtimestamp(base + 0.03))]
    s = clocks.summarize("\n".join(rows), window=(base, base + 0.04))
    assert s["sm_mhz"] == 1965 and s["samples_under_load"] == 2
    # nearest samples outside the window still need the utilisation
    s = clocks.summarize("\n".join(rows), window=(base + 0.1, base + 0.12), slack_s=0.2)
    assert s["samples_in_window"] == 0 and s["sm_mhz"] is None


def test_sampler_left_running_is_stopped_at_exit(tmp_path, monkeypatch):
    """A run that fails between start() and stop(): the exit hook ends exactly the
    sampler's own process (a stand-in nvidia-smi that would sample forever)."""
    import os
    import stat

    from sparknet.utils.clocks import ClockSampler

    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/sh\nwhile true; do echo '0, 1200, 1965, 500.0, 0x0, Not Active, Not Active, Not Active, Not Active'; sleep 0.05; done\n")
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    s = ClockSampler([0], interval_ms=50).start()
    proc, name = s._proc, s._file.name
    assert proc is not None and proc.poll() is None
    s._abandon()          # what atexit runs
    assert proc.poll() is not None and not os.path.exists(name)
    s2 = ClockSampler([0], interval_ms=50).start()
    result = s2.stop()    # the normal path still works and unregisters the hook
    assert result["samples"] >= 0 and s2._proc is None
