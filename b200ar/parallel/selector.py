"""Variant selector: which all-reduce algorithm (and how many CTAs) serves a
message of a given size on a given number of ranks.

The reference switches on one rule only: push when ``bytes * world <= capacity``,
else pull (pcie_allreduce.cu:420-421), and its crossover to NCCL is found by
hand with bench_crossover.py. Here the decision is a table built from
measurements (``build_table`` over per-size latencies, produced by
``bench/allreduce_sweep.py --tune``), loaded per world size and handed to the
native communicator, which applies it identically on every rank. Entries can
name ``nccl``: the measured crossover above which NCCL is faster.
"""

from __future__ import annotations

import json
import math
import os
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

from .._native import _C

VARIANTS: Dict[str, int] = dict(_C.VARIANTS)
VARIANT_NAMES: Dict[int, str] = {v: k for k, v in VARIANTS.items()}

Entry = Tuple[int, str, int]  # (max_bytes, variant name, ctas; 0 = automatic)

_DEFAULT_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "tuning", "b200_nvswitch.json")

# Used when no measured table is available for a world size.
FALLBACK: List[Entry] = [
    (256 << 10, "oneshot_push", 0),
    (1 << 62, "twoshot", 0),
]


def variant_id(name_or_id) -> int:
    if isinstance(name_or_id, int):
        if name_or_id not in VARIANT_NAMES:
            raise ValueError(f"unknown variant id {name_or_id}")
        return name_or_id
    try:
        return VARIANTS[name_or_id]
    except KeyError:
        raise ValueError(f"unknown variant {name_or_id!r}; known: {sorted(VARIANTS)}") from None


def load_table(world: int, path: Optional[str] = None) -> List[Entry]:
    """Returns the selector entries for ``world`` ranks from ``path`` (or the
    packaged table), falling back to ``FALLBACK``."""
    p = path or _DEFAULT_PATH
    if os.path.exists(p):
        with open(p) as f:
            data = json.load(f)
        tables = {int(k): v for k, v in data.get("tables", {}).items() if v}
        if tables:
            # Nearest measured world size on a log scale (ties go to the larger one).
            best = min(tables, key=lambda w: (abs(math.log2(w) - math.log2(max(world, 1))), -w))
            return [(int(b), str(v), int(c)) for b, v, c in tables[best]]
    return list(FALLBACK)


def to_native(entries: Iterable[Entry]) -> List[Tuple[int, int, int]]:
    out = []
    for b, v, c in entries:
        out.append((min(int(b), (1 << 63) - 1), variant_id(v), int(c)))
    return out


def build_table(measurements: Sequence[dict], slack: float = 0.0) -> List[Entry]:
    """Builds a selector table from latency measurements.

    ``measurements``: dicts with keys ``bytes``, ``variant`` (name), ``ctas`` and
    ``us`` (p50 latency). For every size the fastest candidate wins (``slack``
    prefers the candidate listed first when within that relative margin).
    Adjacent sizes with the same winner merge into one entry; each entry covers
    sizes up to and including its largest measured size, the last one covers
    everything above.
    """
    by_size: Dict[int, List[dict]] = {}
    for m in measurements:
        by_size.setdefault(int(m["bytes"]), []).append(m)
    winners: List[Tuple[int, str, int]] = []
    for size in sorted(by_size):
        cands = by_size[size]
        best = min(cands, key=lambda m: m["us"])
        for m in cands:
            if m["us"] <= best["us"] * (1.0 + slack):
                best = m
                break
        winners.append((size, str(best["variant"]), int(best.get("ctas", 0))))
    table: List[Entry] = []
    for size, v, c in winners:
        if table and table[-1][1] == v and table[-1][2] == c:
            table[-1] = (size, v, c)
        else:
            table.append((size, v, c))
    if table:
        last = table[-1]
        table[-1] = (1 << 62, last[1], last[2])
    return table


def merge_partial_table(old: Sequence[Entry], new: Sequence[Entry], min_bytes: int) -> List[Entry]:
    """Table of a sweep that started at ``min_bytes`` (``new``) merged into
    the table of a full sweep (``old``): ``old`` keeps every size below
    ``min_bytes`` (the entry that reached into the new range is cut at
    ``min_bytes // 2``, the last size it was measured at), ``new`` serves the rest."""
    keep: List[Entry] = []
    for b, v, c in old:
        if b < min_bytes:
            keep.append((int(b), str(v), int(c)))
        else:
            keep.append((min_bytes // 2, str(v), int(c)))
            break
    return keep + [(int(b), str(v), int(c)) for b, v, c in new]


def crossover_bytes(measurements: Sequence[dict], ours: str = "custom", theirs: str = "nccl") -> Optional[int]:
    """Smallest size above which ``theirs`` is at least as fast as ``ours`` for
    every larger measured size (None if ours wins everywhere)."""
    sizes = sorted({int(m["bytes"]) for m in measurements})
    best: Dict[Tuple[int, str], float] = {}
    for m in measurements:
        key = (int(m["bytes"]), m["impl"])
        best[key] = min(best.get(key, float("inf")), float(m["us"]))
    cross = None
    for s in reversed(sizes):
        a, b = best.get((s, ours)), best.get((s, theirs))
        if a is None or b is None:
            continue
        if b <= a:
            cross = s
        else:
            break
    return cross


def parity_band(measurements: Sequence[dict], ours: str = "custom", theirs: str = "nccl", lo: float = 0.9,
                hi: float = 1.1) -> List[int]:
    """Sizes whose speedup t_theirs / t_ours lies in [lo, hi]: the reference
    benchmark's crossover marker (bench_crossover.py:207, 232), reported next
    to ``crossover_bytes``."""
    best: Dict[Tuple[int, str], float] = {}
    for m in measurements:
        key = (int(m["bytes"]), m["impl"])
        best[key] = min(best.get(key, float("inf")), float(m["us"]))
    out = []
    for s in sorted({k[0] for k in best}):
        a, b = best.get((s, ours)), best.get((s, theirs))
        if a and b is not None and lo <= b / a <= hi:
            out.append(s)
    return out


def save_tables(path: str, tables: Dict[int, List[Entry]], meta: Optional[dict] = None) -> None:
    data = {"meta": meta or {}, "tables": {str(w): [list(e) for e in t] for w, t in sorted(tables.items())}}
    with open(path, "w") as f:
        json.dump(data, f, indent=1)
