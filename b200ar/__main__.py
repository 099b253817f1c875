"""``python -m b200ar``: prints what b200ar sees on this machine.

The native library and its build, the CUDA devices with their compute
capability, peer access between them and switch multicast (NVLS) support,
the effective configuration (``B200AR_*`` variables) and the selector table
that each world size would use. ``--json`` prints one JSON object instead.
"""

from __future__ import annotations

import argparse
import json
import os
import sys


def collect() -> dict:
    import torch

    from . import _C
    from .config import default_config
    from .parallel.selector import load_table

    info = {
        "library": os.path.basename(_C.__file__),
        "checked_build": _C.__name__.endswith("_checked"),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "config": {k: v for k, v in vars(default_config()).items()},
        "env": {k: v for k, v in sorted(os.environ.items()) if k.startswith("B200AR_")},
        "devices": [],
        "peer_access": [],
        "selector": {str(w): [list(e) for e in load_table(w)] for w in (2, 4, 8)},
    }
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        dev = {"index": i, "name": p.name, "capability": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
               "memory_gib": round(p.total_memory / 2**30, 1)}
        try:
            dev["nvls"] = bool(_C.NvlsBuffer.supported(i))
        except Exception as e:  # noqa: BLE001 - reported, not fatal
            dev["nvls"] = f"unknown ({e})"
        info["devices"].append(dev)
    for i in range(n):
        info["peer_access"].append([i == j or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)])
    return info


def render(info: dict) -> str:
    lines = [f"b200ar native library: {info['library']}" + (" (checked build)" if info["checked_build"] else ""),
             f"torch {info['torch']}, CUDA runtime {info['cuda_runtime']}"]
    if not info["devices"]:
        lines.append("CUDA devices: none visible (the CPU shared-memory backend is available)")
    for d in info["devices"]:
        lines.append(f"  cuda:{d['index']}  {d['name']}  sm_{d['capability'].replace('.', '')}  {d['sms']} SMs  "
                     f"{d['memory_gib']} GiB  NVLS: {d['nvls']}")
    if info["peer_access"]:
        full = all(all(row) for row in info["peer_access"])
        lines.append(f"peer access: {'all pairs' if full else info['peer_access']}")
    lines.append("configuration: " + ", ".join(f"{k}={v}" for k, v in info["config"].items()))
    if info["env"]:
        lines.append("environment: " + ", ".join(f"{k}={v}" for k, v in info["env"].items()))
    for w, table in info["selector"].items():
        lines.append(f"selector, {w} ranks: " + ", ".join(
            f"<= {'inf' if b >= 1 << 62 else b} B: {v}" + (f" ({c} CTAs)" if c else "") for b, v, c in table))
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m b200ar", description=__doc__.splitlines()[0])
    ap.add_argument("--json", action="store_true", help="print one JSON object")
    args = ap.parse_args(argv)
    info = collect()
    print(json.dumps(info) if args.json else render(info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
