"""Per-collective timing trace (``SPARKNET_TRACE=1``) and its offline analysis.

Each rank's runtime maps a file ``/dev/shm/sparknet-trace-r<rank>-p<pid>-<id>.bin``
(header, then a ring of 65536 records of 32 u64 words), pins it for the GPU, and the
collective kernels stamp ``%globaltimer`` into the record of every collective
(indexed by sequence): entry, the arrival of each peer's first pack, and exit.  The
header holds the GPU-minus-host clock offset measured at startup by the clock-probe
kernel (round with the smallest round trip).  Record layout:

    [0] seq | op << 32    [1] bytes    [2] entry ns    [3] exit ns
    [4 + s] arrival of source s's first pack (own entry for s == rank)

The analysis reports per-rank phase distributions (entry -> last arrival, entry ->
exit) and, for every pair of ranks, NTP-style clock offset and one-way delay from
the two directions of each collective.  Reference: ``sparknet/oneshot/trace.py``
(there the host proxy also stamped; here the whole path is on the GPU).
"""

from __future__ import annotations

import argparse
import json
import os
import struct
import sys
import time
import uuid
from pathlib import Path

HEADER_BYTES = 4096
RECORDS = 65536
RECORD_WORDS = 32
RECORD_BYTES = RECORD_WORDS * 8
MAGIC = b"SNTRACE1"
HEADER_FORMAT = "<8sIIIqqqII"  # magic, version, world, rank, offset, halfwidth, created, records, words
VERSION = 1


def enabled(environ=None) -> bool:
    return (environ or os.environ).get("SPARKNET_TRACE", "0") not in ("", "0", "false", "False")


def file_bytes() -> int:
    return HEADER_BYTES + RECORDS * RECORD_BYTES


def pack_header(*, world: int, rank: int, clock_offset_ns: int, clock_halfwidth_ns: int, created_ns: int) -> bytes:
    head = struct.pack(HEADER_FORMAT, MAGIC, VERSION, world, rank, clock_offset_ns, clock_halfwidth_ns, created_ns,
                       RECORDS, RECORD_WORDS)
    return head + b"\0" * (HEADER_BYTES - len(head))


def unpack_header(data: bytes) -> dict:
    magic, version, world, rank, offset, half, created, records, words = struct.unpack_from(HEADER_FORMAT, data)
    if magic != MAGIC:
        raise ValueError("not a sparknet trace file")
    return {"version": version, "world": world, "rank": rank, "clock_offset_ns": offset,
            "clock_halfwidth_ns": half, "created_ns": created, "records": records, "words": words}


def calibrate(samples: list[tuple[int, int, int]]) -> tuple[int, int]:
    """GPU-minus-host offset and its uncertainty from (host_send, gpu, host_recv) rounds:
    the round with the smallest round trip wins (NTP's minimum-delay filter)."""
    if not samples:
        return 0, 0
    t0, g, t1 = min(samples, key=lambda s: s[2] - s[0])
    return int(g - (t0 + t1) // 2), int((t1 - t0) // 2)


def open_trace(*, rank: int, world: int, clock_samples: list[tuple[int, int, int]], directory: str = "/dev/shm"):
    """Create and head a trace file; returns (path, mmap, address)."""
    import ctypes
    import mmap

    path = os.path.join(directory, f"sparknet-trace-r{rank}-p{os.getpid()}-{uuid.uuid4().hex[:8]}.bin")
    size = file_bytes()
    fd = os.open(path, os.O_RDWR | os.O_CREAT | os.O_EXCL, 0o644)
    try:
        os.ftruncate(fd, size)
        mapping = mmap.mmap(fd, size)
    finally:
        os.close(fd)
    offset, half = calibrate(clock_samples)
    mapping[:HEADER_BYTES] = pack_header(world=world, rank=rank, clock_offset_ns=offset, clock_halfwidth_ns=half,
                                         created_ns=time.time_ns())
    address = ctypes.addressof(ctypes.c_char.from_buffer(mapping))
    return path, mapping, address


def read(path: str | Path):
    """(header, records) where records is a [RECORDS, RECORD_WORDS] uint64 numpy array."""
    import numpy as np

    data = Path(path).read_bytes()
    header = unpack_header(data)
    recs = np.frombuffer(data, dtype=np.uint64, offset=HEADER_BYTES,
                         count=header["records"] * header["words"]).reshape(header["records"], header["words"])
    return header, recs


def valid(recs):
    return recs[(recs[:, 2] > 0) & (recs[:, 3] >= recs[:, 2])]


def select(recs, *, min_seq: int = 0, max_seq: int | None = None, nbytes: int | None = None, op: int | None = None):
    """The valid records of a sequence range and, optionally, one payload size or one
    collective (``OP_*`` code of the runtime)."""
    r = valid(recs)
    seq = r[:, 0] & 0xFFFFFFFF
    keep = seq >= min_seq
    if max_seq is not None:
        keep &= seq <= max_seq
    if nbytes is not None:
        keep &= r[:, 1] == nbytes
    if op is not None:
        keep &= (r[:, 0] >> 32) == op
    return r[keep]


def sizes(recs, top: int = 8) -> dict[int, int]:
    """Collective counts of the most frequent payload sizes (bytes), most frequent first."""
    counts: dict[int, int] = {}
    for size in valid(recs)[:, 1].tolist():
        counts[int(size)] = counts.get(int(size), 0) + 1
    return dict(sorted(counts.items(), key=lambda item: -item[1])[:top])


def peer_arrival(record, peer: int) -> int:
    """Nanoseconds from a collective's entry to the arrival of ``peer``'s first pack
    (this rank's clock), or -1 when the record holds no arrival for that peer."""
    arrival, entry = int(record[4 + peer]), int(record[2])
    return arrival - entry if arrival and entry else -1


def _percentiles(values) -> dict:
    import numpy as np

    if len(values) == 0:
        return {}
    v = np.asarray(values, dtype=np.float64)
    return {"n": int(v.size), "p5": float(np.percentile(v, 5)), "p50": float(np.percentile(v, 50)),
            "p95": float(np.percentile(v, 95)), "max": float(v.max())}


def phases(header: dict, recs) -> dict:
    """Microsecond distributions of entry->last peer arrival and entry->exit."""
    r = valid(recs)
    world, rank = header["world"], header["rank"]
    peers = [4 + s for s in range(world) if s != rank]
    out = {"collectives": int(len(r))}
    if len(r) == 0:
        return out
    entry = r[:, 2].astype("int64")
    out["total_us"] = _percentiles((r[:, 3].astype("int64") - entry) / 1000.0)
    if peers:
        arrivals = r[:, peers].astype("int64")
        ok = (arrivals > 0).all(axis=1)
        if ok.any():
            out["wait_us"] = _percentiles((arrivals[ok].max(axis=1) - entry[ok]) / 1000.0)
            out["first_arrival_us"] = _percentiles((arrivals[ok].min(axis=1) - entry[ok]) / 1000.0)
    return out


def pair_clock(a: tuple[dict, object], b: tuple[dict, object]) -> dict:
    """NTP-style offset (b minus a) and one-way delay from collectives both ranks traced.

    For a collective with sequence s: d_ab = arrival at b of a's data (b's clock) minus
    a's entry (a's clock), d_ba likewise; offset = (d_ab - d_ba) / 2, delay = (d_ab +
    d_ba) / 2.  Medians over the common sequences, in microseconds.
    """
    import numpy as np

    (ha, ra), (hb, rb) = a, b
    ia, ib = ha["rank"], hb["rank"]
    va, vb = valid(ra), valid(rb)
    sa = {int(x[0] & 0xFFFFFFFF): x for x in va}
    offs, delays = [], []
    for x in vb:
        s = int(x[0] & 0xFFFFFFFF)
        y = sa.get(s)
        if y is None or x[4 + ia] == 0 or y[4 + ib] == 0:
            continue
        d_ab = int(x[4 + ia]) - int(y[2])
        d_ba = int(y[4 + ib]) - int(x[2])
        offs.append((d_ab - d_ba) / 2000.0)
        delays.append((d_ab + d_ba) / 2000.0)
    if not offs:
        return {"pairs": 0}
    return {"pairs": len(offs), "offset_us": float(np.median(offs)), "delay_us": float(np.median(delays))}


def summarize(paths: list[str], *, min_seq: int = 0, max_seq: int | None = None, nbytes: int | None = None) -> dict:
    traces = [(h, select(r, min_seq=min_seq, max_seq=max_seq, nbytes=nbytes)) for h, r in (read(p) for p in paths)]
    out = {"ranks": {}, "pairs": {}}
    for h, r in traces:
        out["ranks"][h["rank"]] = {"phases": phases(h, r), "clock_offset_ns": h["clock_offset_ns"],
                                   "clock_halfwidth_ns": h["clock_halfwidth_ns"]}
    for i in range(len(traces)):
        for j in range(i + 1, len(traces)):
            key = f"{traces[i][0]['rank']}-{traces[j][0]['rank']}"
            out["pairs"][key] = pair_clock(traces[i], traces[j])
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("files", nargs="+", help="trace files, one per rank")
    p.add_argument("--min-seq", type=int, default=0)
    p.add_argument("--max-seq", type=int)
    p.add_argument("--nbytes", type=int, help="only collectives of this payload size")
    p.add_argument("--last-seq", action="store_true", help="print each file's newest sequence and exit")
    args = p.parse_args(argv)
    if args.last_seq:
        newest = {}
        for path in args.files:
            r = valid(read(path)[1])
            newest[path] = int((r[:, 0] & 0xFFFFFFFF).max()) if len(r) else 0
        print(json.dumps(newest, indent=2))
        return 0
    print(json.dumps(summarize(args.files, min_seq=args.min_seq, max_seq=args.max_seq, nbytes=args.nbytes), indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
