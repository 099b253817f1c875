"""GQA decode attention on the TP8 Llama-3-70B decode shape (8 query heads and
1 KV head of 128 per rank, 2049 cached tokens) at batch 1/8/32/64.

Two timings per batch, both with CUDA events on the launching stream around
one replay of a CUDA graph of calls, per call:
  warm   20 calls on the same cache (L2-warm K/V: the cache of one layer fits
         in the 126 MB L2 at these batches);
  cold   calls rotating over enough distinct caches (like the layers of a
         model) that their total is at least 3x the L2: every call reads its
         K/V from HBM.
The achieved bandwidth counts the K and V bytes the kernel must read.

    python bench/attention_bench.py [--len 2049] [--impl tc,mma]
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
from b200ar.utils.timing import percentile  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--len", type=int, default=2049)
    ap.add_argument("--batches", default="1,8,32,64")
    ap.add_argument("--impl", default="tc,mma", help="comma list of kernels: tc (tcgen05 + TMA), mma (mma.sync)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    peaks = {}
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peaks = json.load(open(p))
    hq, hkv, L = 8, 1, args.len
    for b, impl in ((int(v), i) for v in args.batches.split(",") for i in args.impl.split(",")):
        kv_bytes = 2 * b * L * hkv * 128 * 2
        sets = max(2, min(512, -(-3 * (126 << 20) // kv_bytes)))
        qs, kcs, vcs = [], [], []
        for _ in range(sets):
            qs.append(torch.randn(b, hq, 128, device=dev).to(torch.bfloat16))
            kcs.append(torch.randn(b, L + 16, hkv, 128, device=dev).to(torch.bfloat16))
            vcs.append(torch.randn(b, L + 16, hkv, 128, device=dev).to(torch.bfloat16))
        seq = torch.full((b,), L, dtype=torch.int32, device=dev)
        out = torch.empty(b, hq * 128, dtype=torch.bfloat16, device=dev)
        for _ in range(args.warmup):
            decode_attention(qs[0], kcs[0], vcs[0], seq, hq, hkv, out=out, impl=impl)
        err = (out.float() - ref_decode_attention(qs[0], kcs[0], vcs[0], seq, hq, hkv)).abs().max().item()

        def timed(order):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in order:
                    decode_attention(qs[i], kcs[i], vcs[i], seq, hq, hkv, out=out, impl=impl)
            g.replay()
            torch.cuda.synchronize()
            vals = []
            for _ in range(5):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                vals.append(e0.elapsed_time(e1) * 1e3 / len(order))
            return percentile(vals, 50)

        warm = timed([0] * 20)
        cold = timed([i % sets for i in range(max(20, 2 * sets))])
        row = {"impl": impl, "batch": b, "seq_len": L, "hq": hq, "hkv": hkv, "max_abs_err": round(err, 4),
               "warm_us": round(warm, 2), "cold_us": round(cold, 2), "caches": sets,
               "cold_tbs": round(kv_bytes / (cold * 1e-6) / 1e12, 3)}
        if peaks.get("hbm_gbs"):
            row["cold_frac_of_measured_hbm"] = round(row["cold_tbs"] * 1e3 / peaks["hbm_gbs"], 3)
        print(json.dumps(row), flush=True)
        del qs, kcs, vcs
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
