"""Renders a bench.py JSON line (or a file of them) as markdown tables.

    python bench.py --gpus 8 --json-out run.json ...
    python bench/render_md.py run.json [--reference ref.json] > table.md

One table per result line: per message size the variant the selector chose,
eager and graph p50 (with p10-p90 where recorded), NCCL eager p50, the
speedup over NCCL, busbw and its fraction of NVLink bandwidth. With
``--reference`` (a line printed by ``bench.py --impl reference``) a column
gives the reference's eager p50 and the ratio to it.
"""

from __future__ import annotations

import argparse
import json
from typing import Dict, List, Optional


def load_lines(path: str) -> List[dict]:
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                out.append(json.loads(line))
    return out


def sweep_of(result: dict) -> List[dict]:
    """Per-size rows of a bench line: the detailed ``sweep`` (``--json-out``)
    or, for a printed line, its compact ``rows`` (columns ``rows_cols``)."""
    if "sweep" in result:
        return result["sweep"]
    cols = result.get("rows_cols")
    if not cols:
        return []
    out = []
    for r in result.get("rows", []):
        d = {k: v for k, v in zip(cols, r) if v is not None}
        if result.get("n_gpus", 1) > 1 and d.get("eager_p50_us"):
            n, s = result["n_gpus"], d["bytes"]
            d["busbw_gbs"] = s / (d["eager_p50_us"] * 1e-6) / 1e9 * 2 * (n - 1) / n
            d["busbw_frac_of_nvlink"] = d["busbw_gbs"] / 770.0
        out.append(d)
    return out


def _fmt_us(row: dict, mode: str) -> str:
    st = row.get(f"{mode}_us")
    p50 = row.get(f"{mode}_p50_us")
    if p50 is None:
        return "-"
    if isinstance(st, dict) and "p10" in st and "p90" in st:
        return f"{p50:.2f} ({st['p10']:.2f}-{st['p90']:.2f})"
    return f"{p50:.2f}"


def render(result: dict, reference: Optional[dict] = None) -> str:
    if "unavailable" in result:
        return f"{result.get('impl', '?')}: unavailable ({result['unavailable']})\n"
    ref_by_size: Dict[int, dict] = {}
    if reference:
        ref_by_size = {r["bytes"]: r for r in sweep_of(reference)}
    head = ["bytes", "variant", "eager us p50 (p10-p90)", "graph us p50 (p10-p90)", "NCCL eager us",
            "NCCL / ours", "busbw GB/s", "of NVLink"]
    if ref_by_size:
        head += ["reference eager us", "reference / ours"]
    lines = [
        f"{result.get('impl', 'b200ar')}, {result.get('n_gpus')} GPU(s): {result.get('metric')} = "
        f"{result.get('value')} {result.get('unit', '')}",
        "",
        "| " + " | ".join(head) + " |",
        "|" + "---|" * len(head),
    ]
    for row in sweep_of(result):
        s = row["bytes"]
        eager = row.get("eager_p50_us")
        nccl = row.get("nccl_eager_p50_us")
        cells = [
            str(s),
            str(row.get("variant", "-")),
            _fmt_us(row, "eager"),
            _fmt_us(row, "graph"),
            f"{nccl:.2f}" if nccl is not None else "-",
            f"{nccl / eager:.2f}x" if nccl and eager else "-",
            f"{row['busbw_gbs']:.1f}" if "busbw_gbs" in row else "-",
            f"{row['busbw_frac_of_nvlink']:.2f}" if "busbw_frac_of_nvlink" in row else "-",
        ]
        if ref_by_size:
            r = ref_by_size.get(s)
            re = r.get("eager_p50_us") if r else None
            cells += [f"{re:.2f}" if re else "-", f"{re / eager:.2f}x" if re and eager else "-"]
        lines.append("| " + " | ".join(cells) + " |")
    cross = result.get("crossover_bytes")
    if cross:
        lines += ["", "NCCL crossover (first size from which NCCL is faster): " +
                  ", ".join(f"{k} {v if v is not None else 'none'}" for k, v in cross.items())]
    band = result.get("crossover_band_bytes")
    if band:
        lines += ["NCCL / ours within [0.9, 1.1] (the reference's crossover marker): " +
                  "; ".join(f"{k} {', '.join(str(b) for b in v) or 'none'}" for k, v in band.items())]
    clocks = result.get("clocks")
    if clocks:
        lines += ["", f"SM clock under load: {clocks.get('sm_mhz')} of {clocks.get('sm_max_mhz')} MHz, "
                      f"reasons: {', '.join(clocks.get('reasons', [])) or 'none'}"]
    return "\n".join(lines) + "\n"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("result")
    ap.add_argument("--reference", default="")
    args = ap.parse_args()
    ref = None
    if args.reference:
        refs = [r for r in load_lines(args.reference) if sweep_of(r)]
        ref = refs[-1] if refs else None
    for res in load_lines(args.result):
        print(render(res, ref))


if __name__ == "__main__":
    main()
