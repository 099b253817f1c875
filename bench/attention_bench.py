"""GQA decode attention on the TP8 Llama-3-70B decode shape (8 query heads and
1 KV head of 128 per rank, 2049 cached tokens) at batch 1/8/32/64.

Two timings per batch, both with CUDA events on the launching stream:
  warm   20 calls captured in one CUDA graph, one replay timed (L2-warm K/V:
         the whole cache fits in the 126 MB L2 at these batches);
  cold   one eager call per sample with L2 flushed before it, p50.
The achieved bandwidth counts the K and V bytes the kernel must read.

    python bench/attention_bench.py [--iters 30] [--len 2049]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from b200ar.ops.layers import decode_attention, ref_decode_attention  # noqa: E402
from b200ar.utils.timing import EventTimer, L2Flusher, percentile  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--len", type=int, default=2049)
    ap.add_argument("--batches", default="1,8,32,64")
    ap.add_argument("--impl", default="tc,mma", help="comma list of kernels: tc (tcgen05 + TMA), mma (mma.sync)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    flush = L2Flusher(dev, lead_us=20)
    peaks = {}
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peaks = json.load(open(p))
    hq, hkv, L = 8, 1, args.len
    for b, impl in ((int(v), i) for v in args.batches.split(",") for i in args.impl.split(",")):
        q = torch.randn(b, hq, 128, device=dev).to(torch.bfloat16)
        kc = torch.randn(b, L + 16, hkv, 128, device=dev).to(torch.bfloat16)
        vc = torch.randn_like(kc)
        seq = torch.full((b,), L, dtype=torch.int32, device=dev)
        out = torch.empty(b, hq * 128, dtype=torch.bfloat16, device=dev)
        for _ in range(args.warmup):
            decode_attention(q, kc, vc, seq, hq, hkv, out=out, impl=impl)
        err = (out.float() - ref_decode_attention(q, kc, vc, seq, hq, hkv)).abs().max().item()
        reps = 20
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                decode_attention(q, kc, vc, seq, hq, hkv, out=out, impl=impl)
        g.replay()
        torch.cuda.synchronize()
        warm = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            warm.append(e0.elapsed_time(e1) * 1e3 / reps)
        timer = EventTimer(pool=2 * args.iters)
        for _ in range(args.iters):
            flush()
            timer.start("cold")
            decode_attention(q, kc, vc, seq, hq, hkv, out=out, impl=impl)
            timer.stop("cold")
        cold = percentile(timer.times_ms()["cold"], 50) * 1e3
        kv_bytes = 2 * b * L * hkv * 128 * 2
        row = {"impl": impl, "batch": b, "seq_len": L, "hq": hq, "hkv": hkv, "max_abs_err": round(err, 4),
               "warm_us": round(percentile(warm, 50), 2), "cold_us": round(cold, 2),
               "cold_tbs": round(kv_bytes / (cold * 1e-6) / 1e12, 3)}
        if peaks.get("hbm_gbs"):
            row["cold_frac_of_measured_hbm"] = round(row["cold_tbs"] * 1e3 / peaks["hbm_gbs"], 3)
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
