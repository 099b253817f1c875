"""Device timing helpers: CUDA-event timing, L2 flushing, max-over-ranks
reduction and summary statistics.

The reference timed with host ``time.perf_counter`` around a loop on each rank
and printed rank 0 only (bench_crossover.py:113-134, 203-210). b200ar times each
call with CUDA events on the launching stream and reduces every iteration's time
with a MAX over ranks before taking percentiles.
"""

from __future__ import annotations

import math
from typing import Dict, List, Sequence

import torch
import torch.distributed as dist

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2 of B200


class L2Flusher:
    """Overwrites a buffer larger than L2 so the next kernel starts cold.

    ``lead_us`` first keeps the GPU busy with a spin kernel so that the host
    has enqueued the timed call (and its events) before the GPU reaches it;
    otherwise a short kernel's event time would include host launch overhead.

    With ``align_group`` (an NCCL group), a one-element NCCL all-reduce runs
    first, so that every rank's GPU leaves the flush at about the same time:
    without it, a collective whose ranks finish at different times (a large
    NCCL call, say) skews the start of the next timed call across ranks, and
    the next call's time absorbs that skew.
    """

    def __init__(self, device, nbytes: int = L2_FLUSH_BYTES, lead_us: float = 60.0, sm_mhz: float = 1965.0,
                 align_group=None):
        self.buf = torch.empty(nbytes // 4, dtype=torch.int32, device=device)
        self.cycles = int(lead_us * sm_mhz)
        self.align_group = align_group
        self.token = torch.zeros(1, dtype=torch.float32, device=device) if align_group is not None else None

    def __call__(self) -> None:
        if self.align_group is not None:
            dist.all_reduce(self.token, group=self.align_group)
        if self.cycles:
            torch.cuda._sleep(self.cycles)
        self.buf.fill_(0x5A5A5A5A)


def aligned_start(group, lead_s: float = 0.002) -> None:
    """Host-side start alignment for end-to-end timing: rank 0 picks a
    deadline ``lead_s`` ahead on the host's monotonic clock (shared by every
    process on the node) and each rank busy-waits until it passes, so ranks
    start their timed region within a few microseconds of each other instead
    of the tens of microseconds a barrier's release leaves between them."""
    import time

    t = [time.monotonic() + lead_s if dist.get_rank(group) == 0 else 0.0]
    dist.broadcast_object_list(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    while time.monotonic() < t[0]:
        pass


class EventTimer:
    """Collects (start, end) CUDA event pairs keyed by name; ``times_ms`` syncs
    once and returns every recorded duration. Events come from a pool created
    up front so that recording costs the host as little as possible."""

    def __init__(self, pool: int = 0):
        self.pairs: Dict[str, List] = {}
        self._pool = [torch.cuda.Event(enable_timing=True) for _ in range(pool)]

    def _event(self):
        return self._pool.pop() if self._pool else torch.cuda.Event(enable_timing=True)

    def start(self, key: str):
        e = self._event()
        e.record()
        self.pairs.setdefault(key, []).append([e, None])

    def stop(self, key: str):
        e = self._event()
        e.record()
        self.pairs[key][-1][1] = e

    def times_ms(self) -> Dict[str, List[float]]:
        torch.cuda.synchronize()
        return {k: [a.elapsed_time(b) for a, b in v] for k, v in self.pairs.items()}


def max_over_ranks(values: Sequence[float], device, group=None) -> List[float]:
    """Element-wise MAX of ``values`` over all ranks (identity without a process group)."""
    if not (dist.is_initialized() and dist.get_world_size(group) > 1):
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.tolist()


def percentile(values: Sequence[float], q: float) -> float:
    v = sorted(values)
    if not v:
        return float("nan")
    k = (len(v) - 1) * q / 100.0
    lo, hi = math.floor(k), math.ceil(k)
    return v[lo] + (v[hi] - v[lo]) * (k - lo)


def geomean(values: Sequence[float]) -> float:
    v = [x for x in values if x > 0]
    return math.exp(sum(math.log(x) for x in v) / len(v)) if v else float("nan")


# Measured NVLink peer-copy bandwidth per direction per GPU on B200 HGX boxes
# (GB/s); the denominator of the all-reduce bandwidth fraction.
NVLINK_GBS = 770.0


def latency_stats(samples_us: Sequence[float]) -> Dict[str, float]:
    """p10 / p50 / p90 / max of per-call latencies (already the max over
    ranks of each call), rounded to ns."""
    return {
        "p10": round(percentile(samples_us, 10), 3),
        "p50": round(percentile(samples_us, 50), 3),
        "p90": round(percentile(samples_us, 90), 3),
        "max": round(max(samples_us), 3) if samples_us else float("nan"),
    }


def allreduce_bandwidth(nbytes: int, world: int, us: float, link_gbs: float = NVLINK_GBS) -> Dict[str, float]:
    """nccl-tests conventions: algbw = S / t; busbw = algbw * 2 (N - 1) / N,
    the per-GPU link traffic of a bandwidth-optimal all-reduce. The fraction
    relates busbw to one GPU's NVLink bandwidth per direction."""
    algbw = nbytes / (us * 1e-6) / 1e9
    busbw = algbw * 2 * (world - 1) / world if world > 1 else 0.0
    return {"algbw_gbs": round(algbw, 1), "busbw_gbs": round(busbw, 1),
            "busbw_frac_of_nvlink": round(busbw / link_gbs, 3)}
