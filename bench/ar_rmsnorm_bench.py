"""Benchmark configuration: fused all-reduce + residual add + RMSNorm at the
Llama-3-70B hidden size (8192), T in {1, 8, 32, 128, 512}.

Per rank: partial [T, 8192] ~ N(0,1), residual [T, 8192] ~ N(0,1),
gamma = 1 + 0.01 N(0,1), eps 1e-5. Times (p50 of max over ranks, L2 flushed):
  fused          b200ar one kernel (one-shot push or two-shot by size)
  ours_unfused   b200ar all-reduce, then PyTorch add + RMSNorm
  nccl_torch     NCCL all-reduce, then PyTorch add + RMSNorm
  ref_torch      the reference's all-reduce kernel (unmodified, its own API),
                 then PyTorch add + RMSNorm (even world sizes, when installed)
and the roofline max(all-reduce bytes over NVLink at 770 GB/s, HBM bytes at
the measured copy bandwidth) for the fused kernel.

    python -m torch.distributed.run --nproc-per-node N bench/ar_rmsnorm_bench.py
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
from b200ar.utils.timing import EventTimer, L2Flusher, max_over_ranks, percentile  # noqa: E402
sys.path.insert(0, os.path.join(ROOT, "bench"))
from reference_arm import ReferenceArm, reference_available  # noqa: E402

NVLINK_GBS = 770.0


def torch_norm(z, gamma, eps):
    zf = z.float()
    return (zf * torch.rsqrt(zf.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()).to(z.dtype)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,8,32,128,512")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29543")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local))
    gloo = dist.new_group(backend="gloo")
    dev = torch.device("cuda", local)
    comm = CustomAllreduce(group=gloo, device=dev, nccl_group=dist.group.WORLD, max_size=80 << 20)
    peaks = {"hbm_gbs": 6650.0}
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peaks = json.load(open(p))
    flush = L2Flusher(dev, align_group=dist.group.WORLD)
    H, eps = 8192, 1e-5
    ref = None
    if world > 1 and world % 2 == 0 and reference_available():
        ref = ReferenceArm(rank, world, gloo, max(int(t) for t in args.tokens.split(",")) * H * 2)
    g0 = torch.Generator(device=dev).manual_seed(7)
    gamma = (1 + 0.01 * torch.randn(H, generator=g0, device=dev)).to(torch.bfloat16)
    for T in (int(t) for t in args.tokens.split(",")):
        g = torch.Generator(device=dev).manual_seed(1234 + rank + T)
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        res = torch.randn(T, H, generator=torch.Generator(device=dev).manual_seed(55), device=dev).to(torch.bfloat16)
        y = torch.empty_like(x)
        z = torch.empty_like(x)
        tmp = torch.empty_like(x)

        def unfused_ours():
            comm.all_reduce(x, out=tmp)
            zz = (tmp.float() + res.float()).to(torch.bfloat16)
            return torch_norm(zz, gamma, eps), zz

        def unfused_nccl():
            tmp.copy_(x)
            dist.all_reduce(tmp)
            zz = (tmp.float() + res.float()).to(torch.bfloat16)
            return torch_norm(zz, gamma, eps), zz

        def unfused_ref():
            ref.all_reduce(x, tmp)
            zz = (tmp.float() + res.float()).to(torch.bfloat16)
            return torch_norm(zz, gamma, eps), zz

        impls = {
            "fused": lambda: comm.all_reduce_residual_rmsnorm(x, res, gamma, eps, out=y, residual_out=z),
            "ours_unfused": unfused_ours,
            "nccl_torch": unfused_nccl,
        }
        if ref is not None:
            impls["ref_torch"] = unfused_ref
        timer = EventTimer(pool=2 * len(impls) * args.iters)
        for it in range(args.warmup + args.iters):
            for name, fn in impls.items():
                flush()
                if it >= args.warmup:
                    timer.start(name)
                fn()
                if it >= args.warmup:
                    timer.stop(name)
        t = timer.times_ms()
        comm.check()
        nbytes = T * H * 2
        t_link = (world - 1) * nbytes / (NVLINK_GBS * 1e9) if world > 1 else 0.0
        t_hbm = 5 * nbytes / (peaks["hbm_gbs"] * 1e9)  # read x, residual; write y, z; stage copy
        roof_us = max(t_link, t_hbm) * 1e6
        row = {"T": T, "hidden": H, "world": world, "roofline_us": round(roof_us, 2)}
        for name, vals in t.items():
            us = percentile(max_over_ranks(vals, dev), 50) * 1e3
            row[f"{name}_us"] = round(us, 2)
        row["fused_frac_of_roofline"] = round(roof_us / row["fused_us"], 3)
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
