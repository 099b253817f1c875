"""A few eager calls of the tcgen05 decode attention on one TP8 decode shape
(8 query heads, 1 KV head of 128, 2049 cached tokens), for a profiler
capture of one launch:

    ncu --set full --clock-control none -k regex:attn_tc -s 2 -c 1 \\
        python bench/profile_attention.py --batch 64
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from b200ar.ops.gemm import check_errors  # noqa: E402
from b200ar.ops.layers import decode_attention  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--len", type=int, default=2049)
    ap.add_argument("--calls", type=int, default=4)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    b, hq, hkv, L = args.batch, 8, 1, args.len
    q = torch.randn(b, hq, 128, device=dev).to(torch.bfloat16)
    kc = torch.randn(b, L + 16, hkv, 128, device=dev).to(torch.bfloat16)
    vc = torch.randn(b, L + 16, hkv, 128, device=dev).to(torch.bfloat16)
    seq = torch.full((b,), L, dtype=torch.int32, device=dev)
    out = torch.empty(b, hq * 128, dtype=torch.bfloat16, device=dev)
    for _ in range(args.calls):
        decode_attention(q, kc, vc, seq, hq, hkv, out=out, impl="tc")
    torch.cuda.synchronize()
    check_errors()
    print("ok", float(out.float().abs().sum()))


if __name__ == "__main__":
    main()
