"""Headline benchmark: bf16 sum all-reduce p50 latency vs message size.

Headline metric: "bf16 allreduce p50 µs vs size at 2/4/8 GPU vs ref
kernel+NCCL; crossover size". Sizes 4 KB .. 256 MB (powers of two), bf16 values
uniform[-1, 1] seeded 1234 + rank, eager and CUDA-graph modes.

One step = one all-reduce of every size in eager mode and one graph replay of
every size, each preceded by an L2 flush (a 256 MiB write) and timed with its
own pair of CUDA events; our arm also times NCCL the same way. Per-call times
are reduced with a MAX over ranks, then p50 over the K steps. ``value`` is the
geometric mean over sizes of the eager p50 (µs, lower is better); the line ends
with compact per-size ``rows`` (columns ``rows_cols``). ``e2e`` times
the public API end to end on the host clock: H2D copy of the input from pinned
memory, all-reduce, D2H copy of the result, synchronize.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200ar|reference]

For N > 1 launch with ``torch.distributed.run --nproc-per-node N``.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "bf16 allreduce p50 µs vs size at 2/4/8 GPU vs ref kernel+NCCL; crossover size"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200ar", "reference"], default="b200ar")
    ap.add_argument("--min-bytes", type=int, default=4 << 10)
    ap.add_argument("--max-bytes", type=int, default=256 << 20)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--json-out", default="")
    return ap.parse_args()


def sizes(lo, hi):
    out, b = [], lo
    while b <= hi:
        out.append(b)
        b *= 2
    return out


def init_dist(n):
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local))
    gloo = dist.new_group(backend="gloo")
    return rank, world, local, gloo


# --------------------------------------------------------------------------- arms
sys.path.insert(0, os.path.join(ROOT, "bench"))
from reference_arm import ReferenceArm  # noqa: E402  (the unmodified reference through its own API)


class OursArm:
    """b200ar through its public API (CustomAllreduce)."""

    name = "b200ar"

    def __init__(self, rank, world, gloo, max_bytes):
        sys.path.insert(0, ROOT)
        from b200ar import CustomAllreduce

        # No NVLS multicast buffer: the selector tables never pick NVLS, and a
        # rank that died with memory bound to a multicast object would fault
        # its peers' GPUs.
        self.comm = CustomAllreduce(group=gloo, device=torch.device("cuda", torch.cuda.current_device()),
                                    nccl_group=dist.group.WORLD, max_size=max_bytes, enable_nvls=False)

    def all_reduce(self, inp, out):
        self.comm.all_reduce(inp, out)

    def post_capture(self):
        pass

    def launches(self):
        return self.comm.launches

    def variant(self, nbytes):
        return self.comm.plan(nbytes)[0]

    def close(self):
        self.comm.close()


# --------------------------------------------------------------------------- measurement
def make_inputs(sz_list, rank, device):
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    inps, outs = {}, {}
    for s in sz_list:
        n = s // 2
        inps[s] = (torch.rand(n, generator=g, device=device, dtype=torch.float32) * 2 - 1).to(torch.bfloat16)
        outs[s] = torch.empty_like(inps[s])
    return inps, outs


def validate(arm, inps, outs, sz_list):
    """Checks each size once against an fp32 NCCL sum (relative tolerance of bf16)."""
    for s in sz_list:
        arm.all_reduce(inps[s], outs[s])
        ref = inps[s].float()
        dist.all_reduce(ref)
        err = (outs[s].float() - ref).abs().max().item()
        tol = 1e-2 * max(1.0, ref.abs().max().item())
        if not err <= tol:
            raise RuntimeError(f"{arm.name}: all-reduce of {s} bytes is wrong (max abs err {err:.3g} > {tol:.3g})")
    torch.cuda.synchronize()


def capture_graphs(fn_by_size, sz_list):
    graphs = {}
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for sz in sz_list:
            fn_by_size(sz)  # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for sz in sz_list:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn_by_size(sz)
        graphs[sz] = g
    torch.cuda.synchronize()
    return graphs


def summarize(per_call, sz_list, world, variant_of, graphs_on, nccl_on, nccl_graphs_on):
    """Per-size rows, the headline value and the crossover fields from
    per-call latencies in us (each already the max over ranks), keyed
    ``<mode>/<bytes>`` with modes eager, graph, nccl_eager and nccl_graph."""
    from b200ar.parallel.selector import crossover_bytes, parity_band
    from b200ar.utils.timing import allreduce_bandwidth, geomean, latency_stats, percentile

    p50 = {key: percentile(v, 50) for key, v in per_call.items()}
    stats = {key: latency_stats(v) for key, v in per_call.items()}
    sweep = []
    cross_rows = {"eager": [], "graph": []}
    for s in sz_list:
        row = {"bytes": s, "variant": variant_of(s), "eager_p50_us": round(p50[f"eager/{s}"], 3)}
        if graphs_on:
            row["graph_p50_us"] = round(p50[f"graph/{s}"], 3)
        if nccl_on:
            row["nccl_eager_p50_us"] = round(p50[f"nccl_eager/{s}"], 3)
            if nccl_graphs_on:
                row["nccl_graph_p50_us"] = round(p50[f"nccl_graph/{s}"], 3)
        row["eager_us"] = stats[f"eager/{s}"]
        if graphs_on:
            row["graph_us"] = stats[f"graph/{s}"]
        if world > 1:
            row.update(allreduce_bandwidth(s, world, p50[f"eager/{s}"]))
        sweep.append(row)
        for mode in ("eager", "graph"):
            if f"{mode}/{s}" in p50 and f"nccl_{mode}/{s}" in p50:
                cross_rows[mode] += [
                    {"bytes": s, "impl": "custom", "us": p50[f"{mode}/{s}"]},
                    {"bytes": s, "impl": "nccl", "us": p50[f"nccl_{mode}/{s}"]},
                ]
    value = round(geomean([r["eager_p50_us"] for r in sweep]), 3)
    cross = {}
    if nccl_on:
        cross["crossover_bytes"] = {m: crossover_bytes(r) for m, r in cross_rows.items() if r}
        cross["crossover_band_bytes"] = {m: parity_band(r) for m, r in cross_rows.items() if r}
    return sweep, value, cross


E2E_REPS = 5  # e2e samples per step of each message up to 1 MiB

ROW_COLS = ["bytes", "variant", "eager_p50_us", "graph_p50_us", "nccl_eager_p50_us", "nccl_graph_p50_us",
            "e2e_p50_us"]


def compact_rows(sweep, e2e_p50=None):
    """One short list per size (columns ``ROW_COLS``; None where a mode did not
    run), so that every size fits in the tail of the printed line."""
    rows = []
    for r in sweep:
        e = (e2e_p50 or {}).get(r["bytes"])
        rows.append([r["bytes"], r["variant"]] + [r.get(k) for k in ROW_COLS[2:6]] +
                    [round(e, 2) if e is not None else None])
    return rows


def run(args):
    sys.path.insert(0, ROOT)
    from b200ar.utils.clocks import ClockSampler
    from b200ar.utils.timing import EventTimer, L2Flusher, aligned_start, geomean, max_over_ranks, percentile

    rank, world, local, gloo = init_dist(args.gpus)
    dev = torch.device("cuda", local)
    sz_list = sizes(args.min_bytes, args.max_bytes)
    arm = (OursArm if args.impl == "b200ar" else ReferenceArm)(rank, world, gloo, args.max_bytes)
    inps, outs = make_inputs(sz_list, rank, dev)
    validate(arm, inps, outs, sz_list)
    flush = L2Flusher(dev, align_group=dist.group.WORLD if world > 1 else None)
    with_nccl = args.impl == "b200ar" and world > 1
    nccl_bufs = {s: inps[s].clone() for s in sz_list} if with_nccl else {}

    graphs, nccl_graphs = {}, {}
    if not args.no_graph:
        graphs = capture_graphs(lambda s: arm.all_reduce(inps[s], outs[s]), sz_list)
        arm.post_capture()
        if with_nccl:
            nccl_graphs = capture_graphs(lambda s: dist.all_reduce(nccl_bufs[s]), sz_list)

    def step(timer):
        for s in sz_list:
            flush()
            timer.start(f"eager/{s}")
            arm.all_reduce(inps[s], outs[s])
            timer.stop(f"eager/{s}")
            if graphs:
                flush()
                timer.start(f"graph/{s}")
                graphs[s].replay()
                timer.stop(f"graph/{s}")
            if with_nccl:
                flush()
                timer.start(f"nccl_eager/{s}")
                dist.all_reduce(nccl_bufs[s])
                timer.stop(f"nccl_eager/{s}")
                if nccl_graphs:
                    flush()
                    timer.start(f"nccl_graph/{s}")
                    nccl_graphs[s].replay()
                    timer.stop(f"nccl_graph/{s}")

    for _ in range(args.warmup):
        step(EventTimer())
    torch.cuda.synchronize()

    # ---- timed region: exactly K steps, barrier + synchronize on both sides ----
    n_keys = len(sz_list) * (1 + bool(graphs)) * (1 + with_nccl)
    timer = EventTimer(pool=2 * n_keys * args.steps)
    dist.barrier()
    torch.cuda.synchronize()
    launches0 = arm.launches()
    sampler = ClockSampler(gpus=",".join(str(i) for i in range(world))) if local == 0 else contextlib.nullcontext()
    with sampler:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            step(timer)
        t1.record()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
    # Eager launches counted by the library plus one kernel per graph replay.
    launches = arm.launches() - launches0 + args.steps * len(graphs)
    total_ms = max_over_ranks([t0.elapsed_time(t1)], dev)[0]
    times = timer.times_ms()
    per_call = {key: [v * 1e3 for v in max_over_ranks(vals, dev)] for key, vals in times.items()}  # µs
    clocks = sampler.summary() if local == 0 else {}

    # ---- end to end through the public API: pinned H2D, all-reduce, D2H ----
    e2e, e2e_p50 = None, None
    if not args.no_e2e:
        host_in = {s: inps[s].cpu().pin_memory() for s in sz_list}
        host_out = {s: torch.empty_like(host_in[s]).pin_memory() for s in sz_list}
        dev_in = {s: torch.empty_like(inps[s]) for s in sz_list}
        e2e_times = {s: [] for s in sz_list}
        # Small messages are sampled E2E_REPS times per step: their e2e time is
        # tens of microseconds of host-side jitter around a short kernel.
        reps = {s: E2E_REPS if s <= (1 << 20) else 1 for s in sz_list}
        for it in range(args.warmup + args.steps):
            for s in (s for s in sz_list for _ in range(reps[s])):
                flush()
                torch.cuda.synchronize()
                if world > 1:
                    aligned_start(gloo)
                t = time.perf_counter()
                dev_in[s].copy_(host_in[s], non_blocking=True)
                arm.all_reduce(dev_in[s], outs[s])
                host_out[s].copy_(outs[s], non_blocking=True)
                torch.cuda.synchronize()
                if it >= args.warmup:
                    e2e_times[s].append((time.perf_counter() - t) * 1e6)
        e2e_p50 = {s: percentile(max_over_ranks(e2e_times[s], dev), 50) for s in sz_list}
        e2e = {
            "value": round(geomean(list(e2e_p50.values())), 3),
            "unit": "us (geomean over sizes of p50, host clock, max over ranks)",
            "h2d_bytes_per_step": int(sum(s * reps[s] for s in sz_list)),
            "d2h_bytes_per_step": int(sum(s * reps[s] for s in sz_list)),
        }

    sweep, value, cross = summarize(per_call, sz_list, world, arm.variant, bool(graphs), with_nccl,
                                    bool(nccl_graphs))
    result = {
        "metric": METRIC,
        "value": value,
        "unit": "us (geomean over sizes of per-size p50, device time, max over ranks)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: uniform[-1,1] seeded 1234+rank",
        "config": {
            "model": "bf16 sum all-reduce sweep",
            "global_batch": len(sz_list),
            "seq_len": None,
            "parallelism": f"tp{world}",
            "sizes_bytes": [sz_list[0], sz_list[-1]],
            "modes": ["eager"] + (["graph"] if graphs else []),
            "l2": "flushed (256 MiB write) before every timed call",
            "alignment": "one-element NCCL all-reduce before each flush (device); e2e starts at a shared "
                         "host-clock deadline (host)",
        },
        "impl": arm.name,
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    result.update(cross)
    if e2e:
        result["e2e"] = e2e
    # Per-size rows last and compact, so that the end of the line (what a
    # log tail keeps) holds every size; p10/p90/max and bandwidths go to --json-out.
    result["rows_cols"] = ROW_COLS
    result["rows"] = compact_rows(sweep, e2e_p50)
    arm.close()
    if rank == 0:
        print(json.dumps(result), flush=True)
        if args.json_out:
            with open(args.json_out, "w") as f:
                f.write(json.dumps(dict(result, sweep=sweep)) + "\n")
    # Orderly teardown: captured graphs first (some hold NCCL work), then the
    # device, then the process groups; the interpreter then exits normally.
    graphs.clear()
    nccl_graphs.clear()
    torch.cuda.synchronize()
    dist.barrier(group=gloo)
    dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference" and args.gpus < 2:
        print(json.dumps({"impl": "reference", "metric": METRIC,
                          "unavailable": "the reference supports world sizes 2, 4, 6 and 8 only "
                                         "(init_custom_ar rejects odd world sizes, pcie_allreduce.cu:493)"}))
        return
    run(args)


if __name__ == "__main__":
    main()
