"""A few eager calls of b200ar's bf16 linear (x [M, K] @ W [N, K]^T) on one
shape, for a profiler capture of one launch:

    ncu --set full --clock-control none -k regex:skinny -s 2 -c 1 \\
        python bench/profile_gemm.py --shape 1x7168x8192
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from b200ar.ops.gemm import check_errors, linear  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="1x7168x8192", help="MxNxK")
    ap.add_argument("--calls", type=int, default=4)
    args = ap.parse_args()
    m, n, k = (int(v) for v in args.shape.split("x"))
    dev = torch.device("cuda", 0)
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=dev)).to(torch.bfloat16)
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    for _ in range(args.calls):
        linear(x, w, out=out)
    torch.cuda.synchronize()
    check_errors()
    ref = x.float() @ w.float().t()
    print("ok", float((out.float() - ref).abs().max()))


if __name__ == "__main__":
    main()
