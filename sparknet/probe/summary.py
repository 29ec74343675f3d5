"""Latency tables from probe receipts.

Behaviour follows the reference's ``sparknet/probe/summary.py`` (its tables: one per
operation, sizes down, one column per labelled run, deltas against the first).  The
code is this package's own: receipts are read into ``CaseKey``-indexed sample
matrices and reduced with one pass per case.

A receipt is one box's JSON result from ``sparknet probe collectives --benchmark``:
``{"timings": [row, ...]}`` where every row carries ``operation``, ``dtype``,
``elements_per_rank``, an optional ``arm`` (``policy`` when absent) and
``microseconds_per_call``, a list of samples each already the slowest rank of that
box.  Several boxes of one job are combined sample by sample (the slowest box per
sample), and the case's number is the median of that series.
"""

from __future__ import annotations

import json
import statistics
from pathlib import Path
from typing import Iterable, Mapping, NamedTuple

# bytes per element for the dtype names a receipt may carry (``torch.`` prefix optional)
ITEM_SIZES = {"bfloat16": 2, "float16": 2, "float32": 4, "float64": 8, "int8": 1, "uint8": 1, "int32": 4, "int64": 8}
# table order; operations outside it follow in name order
OPERATIONS = ("all_reduce", "all_gather", "reduce_scatter", "fused_norm")


class CaseKey(NamedTuple):
    operation: str
    dtype: str
    nbytes: int
    arm: str


def _bare_dtype(name: object) -> str:
    text = str(name)
    return text.split(".", 1)[1] if text.startswith("torch.") else text


def payload_bytes(row: Mapping) -> int:
    """Bytes per rank of one timing row (elements per rank times the element size)."""
    dtype = _bare_dtype(row["dtype"])
    if dtype not in ITEM_SIZES:
        raise ValueError(f"timing row has an unknown dtype {row['dtype']!r}")
    return ITEM_SIZES[dtype] * int(row["elements_per_rank"])


def size_label(nbytes: int) -> str:
    """The largest binary unit that divides ``nbytes`` exactly: ``2 MiB``, ``60 KiB``, ``100 B``."""
    value, unit = nbytes, "B"
    for next_unit in ("KiB", "MiB"):
        if value and value % 1024 == 0:
            value, unit = value // 1024, next_unit
        else:
            break
    return f"{value} {unit}"


def load_results(directory: str | Path) -> dict[str, dict]:
    """Every ``<box>.json`` under ``directory`` that holds a ``timings`` list, by box name.

    Other JSON files (plans, logs) are skipped; a directory with no receipt at all is
    an error, so a fleet run that produced nothing does not print an empty table."""
    found: dict[str, dict] = {}
    for path in sorted(Path(directory).glob("*.json")):
        body = json.loads(path.read_text())
        if isinstance(body, dict) and isinstance(body.get("timings"), list):
            found[path.stem] = body
    if not found:
        raise FileNotFoundError(f"{directory}: no probe receipt (a <box>.json holding a 'timings' list)")
    return found


def _samples_by_case(results: Mapping[str, Mapping]) -> dict[CaseKey, dict[str, list[float]]]:
    matrix: dict[CaseKey, dict[str, list[float]]] = {}
    for box, receipt in results.items():
        for row in receipt.get("timings", ()):
            key = CaseKey(row["operation"], _bare_dtype(row["dtype"]), payload_bytes(row), row.get("arm") or "policy")
            matrix.setdefault(key, {})[box] = [float(v) for v in row["microseconds_per_call"]]
    return matrix


def cases(results: Mapping[str, Mapping]) -> dict[CaseKey, dict]:
    """Per case: the median over samples of the slowest box, plus each box's own median.

    Boxes with fewer samples than the others limit the series to the common length."""
    table: dict[CaseKey, dict] = {}
    for key, per_box in _samples_by_case(results).items():
        series = list(zip(*per_box.values()))  # one tuple per sample index, one entry per box
        table[key] = {
            "slowest_rank_median_us": statistics.median(max(sample) for sample in series),
            "box_median_us": {box: statistics.median(values) for box, values in per_box.items()},
            "boxes": len(per_box),
            "samples": len(series),
        }
    return table


def _table_order(keys: Iterable[tuple[str, str]]) -> list[tuple[str, str]]:
    rank = {op: i for i, op in enumerate(OPERATIONS)}
    return sorted(set(keys), key=lambda oa: (rank.get(oa[0], len(rank)), oa[0], oa[1]))


def markdown(labelled: Mapping[str, Mapping[CaseKey, dict]], *, dtype: str = "bfloat16") -> str:
    """Markdown tables, one per (operation, arm): a row per message size, a column per
    label; every column after the first shows its change against the first label."""
    labels = list(labelled)
    if not labels:
        return "\n"
    present = [k for table in labelled.values() for k in table if k[1] == dtype]
    out: list[str] = []
    for operation, arm in _table_order((k[0], k[3]) for k in present):
        title = f"{operation.replace('_', '-')} [{arm}] ({dtype}), per rank"
        columns = [labels[0]] + [f"{label} (vs {labels[0]})" for label in labels[1:]]
        out.append("| " + " | ".join([title, *columns]) + " |")
        out.append("| --- |" + " ---: |" * len(labels))
        for nbytes in sorted({k[2] for k in present if k[0] == operation and k[3] == arm}):
            key = CaseKey(operation, dtype, nbytes, arm)
            first = labelled[labels[0]].get(key)
            cells = [size_label(nbytes)]
            for position, label in enumerate(labels):
                entry = labelled[label].get(key)
                if entry is None:
                    cells.append("")
                    continue
                us = entry["slowest_rank_median_us"]
                cell = f"{us:.1f} us"
                if position and first:
                    base = first["slowest_rank_median_us"]
                    cell += f", {100.0 * (us / base - 1.0):+.1f}%"
                cells.append(cell)
            out.append("| " + " | ".join(cells) + " |")
        out.append("")
    return "\n".join(out).rstrip() + "\n"


__all__ = ["CaseKey", "ITEM_SIZES", "OPERATIONS", "cases", "load_results", "markdown", "payload_bytes",
           "size_label"]
