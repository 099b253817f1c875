"""Benchmark configuration: TP Llama-3-70B-shaped decoder slice, decode step.

8 layers, hidden 8192, 64/8 heads of 128, FFN 28672, KV cache pre-filled with
2048 random tokens, random-init weights; batch 1 / 8 / 32 / 64; both the
b200ar step, the plain-PyTorch step (cuBLAS + NCCL + PyTorch attention) and,
for even world sizes when the reference library is installed, the same
PyTorch step with the reference's all-reduce kernel in place of NCCL
(``torch_refar``) are captured in CUDA graphs and timed with CUDA events (max over
ranks, p50 of replays). Weights (~1.7 GB per rank per step at TP 8) exceed L2.

    python -m torch.distributed.run --nproc-per-node N bench/decoder_bench.py
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
from b200ar.models.llama import LlamaConfig, ReferenceDecoder, TPLlamaDecoder  # noqa: E402
from b200ar.utils.timing import EventTimer, max_over_ranks, percentile  # noqa: E402
sys.path.insert(0, os.path.join(ROOT, "bench"))
from reference_arm import ReferenceArm, reference_available  # noqa: E402


def step_bytes(model) -> int:
    """Bytes one decode step must read from HBM on this rank: every weight
    matrix once, plus the KV cache of every layer up to the current length."""
    w = sum(t.numel() * t.element_size() for L in model.layers for t in L.values())
    kv_per_token = 2 * model.hkv * model.cfg.head_dim * 2 * len(model.layers)
    return w + int(model.seq_len.max().item()) * kv_per_token * model.batch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batches", default="1,8,32,64")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--context", type=int, default=2048)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29541")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local))
    gloo = dist.new_group(backend="gloo")
    dev = torch.device("cuda", local)
    comm = CustomAllreduce(group=gloo, device=dev, nccl_group=dist.group.WORLD, max_size=16 << 20)
    cfg = LlamaConfig.llama3_70b_slice(args.layers)
    ref_ar = None
    if world > 1 and world % 2 == 0 and reference_available():
        max_b = max(int(b) for b in args.batches.split(","))
        ref_ar = ReferenceArm(rank, world, gloo, max_b * cfg.hidden * 2)
    peaks = {}
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peaks = json.load(open(pk))
    for B in (int(b) for b in args.batches.split(",")):
        # Every replay (and each capture's warm-up step) advances the position by
        # one: room for all arms' steps past the prefilled context.
        steps = 3 * (args.warmup + args.iters + 1)
        model = TPLlamaDecoder(comm, cfg, batch=B, max_len=args.context + steps + 8)
        model.prefill_random(args.context)
        model.set_input((torch.randn(B, cfg.hidden, device=dev)).to(torch.bfloat16))
        ours = model.capture()
        ref = ReferenceDecoder(model).capture()
        arms = [("b200ar", ours), ("torch_nccl", ref)]
        if ref_ar is not None:
            tmp = torch.empty(B, cfg.hidden, dtype=torch.bfloat16, device=dev)

            def ref_allreduce(t):  # the reference's API is out of place
                ref_ar.all_reduce(t, tmp)
                t.copy_(tmp)

            arms.append(("torch_refar", ReferenceDecoder(model, allreduce=ref_allreduce).capture()))
            ref_ar.post_capture()
        res = {"batch": B, "world": world, "layers": cfg.layers, "hbm_bytes_per_step": step_bytes(model)}
        for name, g in arms:
            timer = EventTimer(pool=2 * args.iters)
            for it in range(args.warmup + args.iters):
                if it >= args.warmup:
                    timer.start(name)
                g.replay()
                if it >= args.warmup:
                    timer.stop(name)
            ms = percentile(max_over_ranks(timer.times_ms()[name], dev), 50)
            res[f"{name}_ms_per_step"] = round(ms, 4)
            res[f"{name}_tokens_per_s"] = round(B / (ms * 1e-3), 1)
        res["speedup"] = round(res["torch_nccl_ms_per_step"] / res["b200ar_ms_per_step"], 3)
        if peaks.get("hbm_gbs"):
            # Weight and KV streaming at the measured copy bandwidth (a lower
            # bound that ignores the all-reduces and launch gaps).
            bound_ms = res["hbm_bytes_per_step"] / (peaks["hbm_gbs"] * 1e9) * 1e3
            res["hbm_bound_ms"] = round(bound_ms, 4)
            res["b200ar_frac_of_hbm_bound"] = round(bound_ms / res["b200ar_ms_per_step"], 3)
        if rank == 0:
            print(json.dumps(res), flush=True)
        del model, ours, ref, arms
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    comm.close()
    if ref_ar is not None:
        ref_ar.close()
    torch.cuda.synchronize()
    dist.barrier(group=gloo)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
