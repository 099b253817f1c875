"""Per-variant all-reduce sweep and selector tuning.

For every message size, times each b200ar variant over a few CTA counts and
NCCL (eager), with the same method as bench.py (L2 flush + lead spin before
each call, CUDA events, max over ranks, p50). With ``--tune PATH`` the fastest
candidate per size becomes the selector table for this world size (merged into
PATH), including ``nccl`` where NCCL wins: the measured crossover.

    python -m torch.distributed.run --nproc-per-node N bench/allreduce_sweep.py \
        [--tune b200ar/tuning/b200_nvswitch.json] [--out sweep.json]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from b200ar import CustomAllreduce  # noqa: E402
from b200ar.parallel import selector as sel  # noqa: E402
from b200ar.utils.timing import EventTimer, L2Flusher, max_over_ranks, percentile  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-bytes", type=int, default=4 << 10)
    ap.add_argument("--max-bytes", type=int, default=256 << 20)
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tune", default="")
    ap.add_argument("--out", default="")
    ap.add_argument("--nvls", action="store_true")
    ap.add_argument("--variants", default="oneshot_push,oneshot_pull,twoshot,twoshot_push,lamport,nvls",
                    help="comma list of b200ar variants to time (NCCL is always timed)")
    ap.add_argument("--ctas", type=lambda v: [int(x) for x in v.split(",")], default=[1, 2, 4, 8, 16, 32, 64, 148, 296, 444])
    args = ap.parse_args()

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    gloo = dist.new_group(backend="gloo")
    dev = torch.device("cuda", local)
    comm = CustomAllreduce(group=gloo, device=dev, nccl_group=dist.group.WORLD, max_size=args.max_bytes,
                           push_max_size=max(1 << 20, args.max_bytes // 16), lamport_max_size=4 << 20,
                           enable_nvls=args.nvls)
    flush = L2Flusher(dev, align_group=dist.group.WORLD)

    sizes = []
    b = args.min_bytes
    while b <= args.max_bytes:
        sizes.append(b)
        b *= 2

    rows = []
    for s in sizes:
        x = (torch.rand(s // 2, device=dev) * 2 - 1).to(torch.bfloat16)
        y = torch.empty_like(x)
        packets = s // 16
        cands = []
        for v in args.variants.split(","):
            if v in ("oneshot_push", "oneshot_pull", "twoshot", "twoshot_push") and _C_slot(v, s, world) > comm.slot_capacity:
                continue
            if v == "lamport" and s > comm.lamport_capacity:
                continue
            if v == "nvls" and (comm.nvls is None or s > comm.nvls.bytes):
                continue
            per = packets // world if v in ("twoshot", "twoshot_push", "nvls") else packets
            resident = comm._comm.resident_ctas(sel.VARIANTS[v])
            for ctas in args.ctas:
                if ctas > 1 and per // ctas < 32:
                    continue
                if ctas > min(512, resident):  # the launch would be clamped to the co-resident count
                    continue
                cands.append((v, ctas))
        # NCCL as the library runs it out of place (reduce-scatter into the
        # output's shard + in-place all-gather): what a table entry "nccl" costs.
        cands.append(("nccl", 0))
        timer = EventTimer(pool=2 * len(cands) * args.iters)
        for it in range(args.warmup + args.iters):
            for v, c in cands:
                flush()
                if it >= args.warmup:
                    timer.start(f"{v}/{c}")
                if v == "nccl":
                    comm._nccl(x, y)
                else:
                    comm.all_reduce(x, y, variant=v, ctas=c)
                if it >= args.warmup:
                    timer.stop(f"{v}/{c}")
        times = timer.times_ms()
        comm.check()
        for key, vals in times.items():
            v, c = key.split("/")
            us = percentile(max_over_ranks(vals, dev), 50) * 1e3
            rows.append({"bytes": s, "variant": v, "ctas": int(c), "us": us,
                         "impl": "nccl" if v == "nccl" else "custom"})
        if rank == 0:
            best = min((r for r in rows if r["bytes"] == s), key=lambda r: r["us"])
            nccl = [r for r in rows if r["bytes"] == s and r["variant"] == "nccl"][0]
            print(f"{s:>11d}  best {best['variant']:>13s}/{best['ctas']:<3d} {best['us']:9.2f} us   "
                  f"nccl {nccl['us']:9.2f} us", file=sys.stderr, flush=True)

    if rank == 0:
        table = sel.build_table(rows)
        out = {"world": world, "rows": rows, "table": table, "crossover_bytes": sel.crossover_bytes(rows)}
        if args.out:
            with open(args.out, "w") as f:
                json.dump(out, f, indent=1)
        if args.tune:
            tables = {}
            if os.path.exists(args.tune):
                with open(args.tune) as f:
                    tables = {int(k): [tuple(e) for e in v] for k, v in json.load(f).get("tables", {}).items()}
            if args.min_bytes > 4096 and world in tables:
                table = sel.merge_partial_table(tables[world], table, args.min_bytes)
            tables[world] = table
            sel.save_tables(args.tune, tables, {"how": "bench/allreduce_sweep.py, p50 of max over ranks"})
        print(json.dumps({"world": world, "table": table, "crossover_bytes": out["crossover_bytes"]}))
    comm.close()  # releases the NVLS buffer before the process ends
    torch.cuda.synchronize()
    dist.barrier(group=gloo)
    dist.destroy_process_group()


def _C_slot(variant, nbytes, world):
    from b200ar import _C

    return _C.variant_slot_bytes(sel.VARIANTS[variant], nbytes, world)


if __name__ == "__main__":
    main()
