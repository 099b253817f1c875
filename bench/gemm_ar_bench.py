"""Benchmark configuration: TP row-parallel down projection fused with its all-reduce.

Per rank x [M, 3584] ~ N(0,1), W [8192, 3584] ~ N(0, 0.02), M in {16, 128, 1024,
8192}. Times (p50 of max over ranks, L2 flushed before every call):
  fused      one tcgen05 kernel, reduce-scatter pushed from the epilogue
  ours_split tcgen05 GEMM, then the b200ar all-reduce
  cublas_nccl torch.matmul, then NCCL all_reduce
  cublas_ref  torch.matmul, then the reference's all-reduce kernel (unmodified,
              its own API; even world sizes, when installed)
and reports each against the roofline max(FLOPs / measured bf16 peak,
2 (N-1)/N * bytes / 770 GB/s per direction).

    python -m torch.distributed.run --nproc-per-node N bench/gemm_ar_bench.py
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
from b200ar.ops.gemm import check_errors, linear  # noqa: E402
from b200ar.utils.timing import EventTimer, L2Flusher, max_over_ranks, percentile  # noqa: E402
sys.path.insert(0, os.path.join(ROOT, "bench"))
from reference_arm import ReferenceArm, reference_available  # noqa: E402

NVLINK_GBS = 770.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ms", default="16,128,1024,8192")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    gloo = dist.new_group(backend="gloo")
    dev = torch.device("cuda", local)
    comm = CustomAllreduce(group=gloo, device=dev, nccl_group=dist.group.WORLD, max_size=160 << 20)
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {"bf16_tflops": 1590.0}
    flush = L2Flusher(dev, align_group=dist.group.WORLD)
    K, N = 3584, 8192
    rows = []
    ref = None
    if world > 1 and world % 2 == 0 and reference_available():
        ref = ReferenceArm(rank, world, gloo, max(int(v) for v in args.ms.split(",")) * N * 2)
    for m in (int(v) for v in args.ms.split(",")):
        g = torch.Generator(device=dev).manual_seed(1234 + rank + m)
        x = torch.randn(m, K, generator=g, device=dev).to(torch.bfloat16)
        w = (0.02 * torch.randn(N, K, generator=g, device=dev)).to(torch.bfloat16)
        out = torch.empty(m, N, dtype=torch.bfloat16, device=dev)
        part = torch.empty_like(out)
        impls = {
            "fused": lambda: comm.linear_all_reduce(x, w, out=out),
            "ours_split": lambda: comm.all_reduce(linear(x, w, out=part), out=out),
            "cublas_nccl": lambda: dist.all_reduce(torch.matmul(x, w.t(), out=part)),
        }
        if ref is not None:
            impls["cublas_ref"] = lambda: ref.all_reduce(torch.matmul(x, w.t(), out=part), out)
        timer = EventTimer(pool=2 * len(impls) * args.iters)
        for it in range(args.warmup + args.iters):
            for name, fn in impls.items():
                flush()
                if it >= args.warmup:
                    timer.start(name)
                fn()
                if it >= args.warmup:
                    timer.stop(name)
        times = timer.times_ms()
        check_errors()
        comm.check()
        flops = 2.0 * m * N * K
        t_compute = flops / (peaks["bf16_tflops"] * 1e12)
        t_link = 2 * (world - 1) / world * m * N * 2 / (NVLINK_GBS * 1e9)
        roof_us = max(t_compute, t_link) * 1e6
        row = {"M": m, "N": N, "K": K, "world": world, "roofline_us": round(roof_us, 2)}
        for name, vals in times.items():
            us = percentile(max_over_ranks(vals, dev), 50) * 1e3
            row[f"{name}_us"] = round(us, 2)
            row[f"{name}_frac_of_roofline"] = round(roof_us / us, 3)
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
    comm.close()
    if ref is not None:
        ref.close()
    torch.cuda.synchronize()
    dist.barrier(group=gloo)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
