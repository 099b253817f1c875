"""tcgen05 GEMM throughput (single-CTA tiles and, above 128 rows, CTA-pair
tiles) vs cuBLAS (torch.matmul) on the row-parallel
down-projection shapes (x [M, 3584] @ W[8192, 3584]^T, M in {16, 128, 1024, 8192}) plus a
square 8192^3 case. CUDA-event timing, L2 flushed before every call, p50.

    python bench/gemm_bench.py [--iters 50]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from b200ar.ops.gemm import check_errors, linear  # noqa: E402
from b200ar.utils.timing import EventTimer, L2Flusher, percentile  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--shapes", default="1x1280x8192,8x1280x8192,64x1280x8192,1x8192x1024,8x7168x8192,64x7168x8192,8x8192x3584,64x8192x3584,16x8192x3584,128x8192x3584,1024x8192x3584,8192x8192x3584,8192x8192x8192")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    flush = L2Flusher(dev, lead_us=20)
    peaks = {}
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peaks = json.load(open(p))
    rows = []
    for shp in args.shapes.split(","):
        m, n, k = (int(v) for v in shp.split("x"))
        a = torch.randn(m, k, device=dev).to(torch.bfloat16)
        w = (0.02 * torch.randn(n, k, device=dev)).to(torch.bfloat16)
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        names = ("tcgen05", "tcgen05_pair", "cublas") if m >= 64 else ("tcgen05", "cublas")
        timer = EventTimer(pool=2 * len(names) * args.iters)
        for it in range(args.warmup + args.iters):
            for name in names:
                flush()
                if it >= args.warmup:
                    timer.start(name)
                if name == "tcgen05":
                    linear(a, w, out=out, pair=False)
                elif name == "tcgen05_pair":
                    linear(a, w, out=out, skinny=False, pair=True)
                else:
                    torch.matmul(a, w.t(), out=out)
                if it >= args.warmup:
                    timer.stop(name)
        t = timer.times_ms()
        check_errors()
        flops = 2.0 * m * n * k
        row = {"M": m, "N": n, "K": k}
        for name in names:
            us = percentile(t[name], 50) * 1e3
            row[f"{name}_us"] = round(us, 2)
            row[f"{name}_tflops"] = round(flops / (us * 1e-6) / 1e12, 1)
        # Streaming: a CUDA graph of calls rotating over enough weight copies
        # (like the layers of a model) that every call reads its weights from
        # HBM, with no flush between calls (the flush leaves L2 full of dirty
        # lines, which small GEMMs then pay to write back).
        wbytes = n * k * 2
        copies = max(2, min(64, -(-3 * (126 << 20) // wbytes)))
        if copies * wbytes <= (8 << 30):
            ws = [w] + [torch.empty_like(w).copy_(w) for _ in range(copies - 1)]
            for name in ("tcgen05", "cublas"):
                def call(wi, name=name):
                    if name == "tcgen05":
                        linear(a, wi, out=out)  # the default path for this shape
                    else:
                        torch.matmul(a, wi.t(), out=out)
                order = [ws[i % copies] for i in range(max(2 * copies, 16))]
                g = torch.cuda.CUDAGraph()
                call(ws[0])
                torch.cuda.synchronize()
                with torch.cuda.graph(g):
                    for wi in order:
                        call(wi)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                row[f"{name}_stream_us"] = round(e0.elapsed_time(e1) * 1e3 / len(order), 2)
            del ws
            check_errors()
        if peaks.get("bf16_tflops"):
            for name in names[:-1]:
                row[f"{name}_frac_of_measured_peak"] = round(row[f"{name}_tflops"] / peaks["bf16_tflops"], 3)
        # Weight-streaming bound for small M: bytes of A, B and C over measured HBM bandwidth.
        if peaks.get("hbm_gbs"):
            bytes_ = 2 * (m * k + n * k + m * n)
            row["hbm_bound_us"] = round(bytes_ / (peaks["hbm_gbs"] * 1e9) * 1e6, 2)
        rows.append(row)
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
