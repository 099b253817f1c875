"""One rank's share of the TP8 Llama-3-70B decoder step, on one GPU.

Builds the decoder slice with the per-rank shapes of tensor parallelism over 8
GPUs (8 query heads and 1 KV head of 128, FFN 3584, hidden 8192) at world size
1, so every GEMM, attention and norm kernel runs on the shapes it has at TP8;
the two all-reduces per layer become the single-rank fused residual + RMSNorm.
Prints the CUDA-graph step time (warm and with the weights of --copies model
instances rotated so they come from HBM), then runs --eager-steps eager steps,
which a per-kernel launch list can capture:

    ncu --metrics gpu__time_duration.sum --clock-control none --csv \\
        python bench/profile_decoder.py --batch 1 --eager-steps 1
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from b200ar import CustomAllreduce  # noqa: E402
from b200ar.models.llama import LlamaConfig, TPLlamaDecoder  # noqa: E402
from b200ar.ops.gemm import check_errors  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--tp", type=int, default=8, help="tensor-parallel degree whose per-rank shapes to run")
    ap.add_argument("--eager-steps", type=int, default=0)
    ap.add_argument("--no-graph", action="store_true")
    args = ap.parse_args()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    comm = CustomAllreduce(device=dev, max_size=16 << 20)
    full = LlamaConfig.llama3_70b_slice(args.layers)
    cfg = LlamaConfig(hidden=full.hidden, heads=full.heads // args.tp, kv_heads=max(1, full.kv_heads // args.tp),
                      head_dim=full.head_dim, intermediate=full.intermediate // args.tp, layers=args.layers)
    steps = 64 + args.eager_steps
    model = TPLlamaDecoder(comm, cfg, batch=args.batch, max_len=args.context + steps + 8)
    model.prefill_random(args.context)
    model.set_input(torch.randn(args.batch, cfg.hidden, device=dev).to(torch.bfloat16))
    res = {"batch": args.batch, "tp_shapes": args.tp, "layers": args.layers}
    if not args.no_graph:
        g = model.capture()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        times.sort()
        w = sum(t.numel() * t.element_size() for L in model.layers for t in L.values())
        res["graph_ms"] = round(times[len(times) // 2], 4)
        res["weight_bytes"] = w
        res["weights_at_hbm_ms"] = None
        p = os.path.join(ROOT, "MEASURED_PEAKS.json")
        if os.path.exists(p):
            hbm = json.load(open(p))["hbm_gbs"]
            kv = 2 * model.hkv * cfg.head_dim * 2 * cfg.layers * args.batch * (args.context + 1)
            res["weights_at_hbm_ms"] = round((w + kv) / (hbm * 1e9) * 1e3, 4)
            res["frac_of_hbm_bound"] = round(res["weights_at_hbm_ms"] / res["graph_ms"], 3)
    for _ in range(args.eager_steps):
        model.forward_step()
    torch.cuda.synchronize()
    check_errors()
    comm.check()
    print(json.dumps(res), flush=True)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
