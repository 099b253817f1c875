"""Samples SM clocks and throttle reasons with ``nvidia-smi`` while a timed
region runs (read-only: nothing here changes a GPU setting)."""

from __future__ import annotations

import csv
import io
import shutil
import statistics
import subprocess
from typing import Optional

_FIELDS = [
    "index",
    "clocks.sm",
    "clocks.max.sm",
    "power.draw",
    "clocks_event_reasons.active",
    "clocks_event_reasons.hw_slowdown",
    "clocks_event_reasons.hw_thermal_slowdown",
    "clocks_event_reasons.sw_thermal_slowdown",
    "clocks_event_reasons.sw_power_cap",
]
_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """Context manager: ``with ClockSampler() as c: ...; c.summary()``."""

    def __init__(self, interval_ms: int = 200, gpus: Optional[str] = None):
        self.interval_ms = interval_ms
        self.gpus = gpus
        self.proc = None
        self.out = ""

    def __enter__(self):
        exe = shutil.which("nvidia-smi")
        if exe:
            cmd = [exe, f"--query-gpu={','.join(_FIELDS)}", "--format=csv,noheader,nounits", f"-lms={self.interval_ms}"]
            if self.gpus:
                cmd.append(f"--id={self.gpus}")
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                                         bufsize=1)
            # Wait for the first sample so the timed region is covered from its start.
            self.first = self.proc.stdout.readline()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                rest, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                rest, _ = self.proc.communicate()
            self.out = getattr(self, "first", "") + (rest or "")
        return False

    def summary(self) -> dict:
        rows = []
        for rec in csv.reader(io.StringIO(self.out)):
            if len(rec) != len(_FIELDS):
                continue
            try:
                rows.append({"sm": float(rec[1]), "max": float(rec[2]), "flags": [x.strip() for x in rec[5:]]})
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set()
        for r in rows:
            for name, flag in zip(_REASONS, r["flags"]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(r["sm"] for r in rows),
            "sm_max_mhz": max(r["max"] for r in rows),
            "reasons": sorted(reasons),
            "samples": len(rows),
        }
