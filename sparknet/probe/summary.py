"""Latency tables from probe receipts (after the reference's ``sparknet/probe/summary.py``).

A receipt is one box's JSON result from ``sparknet probe collectives --benchmark``.
Each timing row holds samples of microseconds per call, already the slowest rank of
the box per sample; across boxes the slowest box is taken per sample.  The number
for a case is the median of those samples.
"""

from __future__ import annotations

import json
import statistics
from pathlib import Path

ITEM_SIZES = {"bfloat16": 2, "float16": 2, "float32": 4, "float64": 8, "int8": 1, "uint8": 1, "int32": 4, "int64": 8}
OPERATIONS = ("all_reduce", "all_gather", "reduce_scatter", "fused_norm")


def load_results(directory: str | Path) -> dict[str, dict]:
    """Probe receipts (``*.json`` with timings) of a directory, by file stem."""
    results = {}
    for path in sorted(Path(directory).glob("*.json")):
        data = json.loads(path.read_text())
        if isinstance(data, dict) and "timings" in data:
            results[path.stem] = data
    if not results:
        raise FileNotFoundError(f"no probe receipts (<node>.json with timings) under {directory}")
    return results


def dtype_name(value: str) -> str:
    return str(value).replace("torch.", "")


def payload_bytes(row: dict) -> int:
    """Bytes per rank of a timing row."""
    return int(row["elements_per_rank"]) * ITEM_SIZES[dtype_name(row["dtype"])]


def size_label(nbytes: int) -> str:
    """``n MiB`` / ``n KiB`` / ``n B``."""
    for unit, scale in (("MiB", 1 << 20), ("KiB", 1 << 10)):
        if nbytes % scale == 0:
            return f"{nbytes // scale} {unit}"
    return f"{nbytes} B"


def cases(results: dict[str, dict]) -> dict[tuple[str, str, int, str], dict]:
    """Per (operation, dtype, bytes, arm): slowest-box median and each box's median."""
    samples: dict[tuple, dict[str, list[float]]] = {}
    for box, result in results.items():
        for row in result.get("timings", []):
            key = (row["operation"], dtype_name(row["dtype"]), payload_bytes(row), row.get("arm", "policy"))
            samples.setdefault(key, {})[box] = [float(v) for v in row["microseconds_per_call"]]
    table = {}
    for key, by_box in samples.items():
        count = min(len(v) for v in by_box.values())
        slowest = [max(v[i] for v in by_box.values()) for i in range(count)]
        table[key] = {"slowest_rank_median_us": statistics.median(slowest),
                      "box_median_us": {b: statistics.median(v) for b, v in by_box.items()},
                      "boxes": len(by_box), "samples": count}
    return table


def markdown(labelled: dict[str, dict], *, dtype: str = "bfloat16") -> str:
    """One table per (operation, arm): sizes down, one column per label, deltas vs the first label."""
    labels = list(labelled)
    lines = []
    keys = sorted({(k[0], k[3]) for t in labelled.values() for k in t if k[1] == dtype},
                  key=lambda x: (OPERATIONS.index(x[0]) if x[0] in OPERATIONS else 99, x[1]))
    for operation, arm in keys:
        sizes = sorted({k[2] for t in labelled.values() for k in t if k[0] == operation and k[1] == dtype
                        and k[3] == arm})
        header = [f"{operation.replace('_', '-')} [{arm}] ({dtype}), per rank"] + labels[:1] + \
            [f"{label} (vs {labels[0]})" for label in labels[1:]]
        lines.append("| " + " | ".join(header) + " |")
        lines.append("| --- | " + " | ".join("---:" for _ in labels) + " |")
        for nbytes in sizes:
            cells = [size_label(nbytes)]
            base = labelled[labels[0]].get((operation, dtype, nbytes, arm))
            for index, label in enumerate(labels):
                entry = labelled[label].get((operation, dtype, nbytes, arm))
                if entry is None:
                    cells.append("")
                    continue
                value = entry["slowest_rank_median_us"]
                text = f"{value:.1f} us"
                if index and base:
                    text += f", {(value - base['slowest_rank_median_us']) / base['slowest_rank_median_us'] * 100:+.1f}%"
                cells.append(text)
            lines.append("| " + " | ".join(cells) + " |")
        lines.append("")
    return "\n".join(lines).rstrip() + "\n"


__all__ = ["ITEM_SIZES", "OPERATIONS", "cases", "load_results", "markdown", "payload_bytes", "size_label"]
