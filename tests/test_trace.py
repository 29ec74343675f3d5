"""Trace file format and analysis on synthetic files (CPU only), after the reference's
tests/test_trace.py."""

import numpy as np
import pytest

from sparknet.oneshot import trace


def synthetic(tmp_path, rank, world, offset_ns, seqs, delay_ns=1500):
    path = tmp_path / f"r{rank}.bin"
    data = bytearray(trace.file_bytes())
    data[:trace.HEADER_BYTES] = trace.pack_header(world=world, rank=rank, clock_offset_ns=offset_ns,
                                                  clock_halfwidth_ns=200, created_ns=1)
    recs = np.frombuffer(data, dtype=np.uint64, offset=trace.HEADER_BYTES).reshape(trace.RECORDS, trace.RECORD_WORDS)
    for s in seqs:
        entry = 1_000_000 * s + offset_ns          # every rank enters at the same true time
        rec = recs[s % trace.RECORDS]
        rec[0] = s | (1 << 32)
        rec[1] = 10240
        rec[2] = entry
        for src in range(world):
            rec[4 + src] = entry if src == rank else entry + delay_ns
        rec[3] = entry + 4000
    path.write_bytes(bytes(data))
    return str(path)


def test_header_round_trip():
    h = trace.unpack_header(trace.pack_header(world=8, rank=3, clock_offset_ns=-5, clock_halfwidth_ns=7,
                                              created_ns=9))
    assert (h["world"], h["rank"], h["clock_offset_ns"], h["clock_halfwidth_ns"]) == (8, 3, -5, 7)
    with pytest.raises(ValueError):
        trace.unpack_header(b"X" * 64)


def test_calibration_uses_smallest_round_trip():
    samples = [(0, 1000, 100), (200, 1260, 240), (500, 2000, 900)]
    assert trace.calibrate(samples) == (1260 - 220, 20)


def test_phases_and_pair_clock(tmp_path):
    a = synthetic(tmp_path, 0, 2, 0, range(1, 101))
    b = synthetic(tmp_path, 1, 2, 700_000, range(1, 101))
    ta, tb = trace.read(a), trace.read(b)
    ph = trace.phases(*ta)
    assert ph["collectives"] == 100
    assert ph["wait_us"]["p50"] == pytest.approx(1.5) and ph["total_us"]["p50"] == pytest.approx(4.0)
    pc = trace.pair_clock(ta, tb)
    assert pc["pairs"] == 100
    assert pc["offset_us"] == pytest.approx(700.0) and pc["delay_us"] == pytest.approx(1.5)
    summary = trace.summarize([a, b])
    assert summary["pairs"]["0-1"]["pairs"] == 100


def test_enabled_flag():
    assert trace.enabled({"SPARKNET_TRACE": "1"}) and not trace.enabled({"SPARKNET_TRACE": "0"})
    assert not trace.enabled({})


def test_select_sizes_and_peer_arrival(tmp_path):
    path = synthetic(tmp_path, 0, 4, 0, range(1, 41), delay_ns=2500)
    header, recs = trace.read(path)
    recs = recs.copy()
    recs[(np.arange(trace.RECORDS) % 4 == 0) & (recs[:, 2] > 0), 1] = 491520   # every 4th collective is larger
    assert len(trace.select(recs)) == 40
    assert len(trace.select(recs, min_seq=11, max_seq=20)) == 10
    assert len(trace.select(recs, nbytes=491520)) == 10 and len(trace.select(recs, op=1)) == 40
    assert len(trace.select(recs, op=2)) == 0
    assert trace.sizes(recs) == {10240: 30, 491520: 10}
    r = trace.select(recs, min_seq=5, max_seq=5)[0]
    assert trace.peer_arrival(r, 2) == 2500 and trace.peer_arrival(r, 0) == 0
    r[4 + 3] = 0
    assert trace.peer_arrival(r, 3) == -1


def test_cli_selection_and_last_seq(tmp_path, capsys):
    import json

    a = synthetic(tmp_path, 0, 2, 0, range(1, 51))
    b = synthetic(tmp_path, 1, 2, 300_000, range(1, 51))
    assert trace.main([a, b, "--min-seq", "21", "--max-seq", "30"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["ranks"]["0"]["phases"]["collectives"] == 10 and out["pairs"]["0-1"]["pairs"] == 10
    assert trace.main([a, b, "--nbytes", "999"]) == 0
    assert json.loads(capsys.readouterr().out)["ranks"]["1"]["phases"]["collectives"] == 0
    assert trace.main([a, "--last-seq"]) == 0
    assert json.loads(capsys.readouterr().out) == {a: 50}
