"""Runs every single-GPU b200ar kernel once on a TP8-decode-sized case, for
`ncu` captures (one launch per kernel after a warm-up pass):

    python bench/profile_kernels.py                      # plain run
    ncu --set full --clock-control none -k regex:"<kernel>" -s <n> -c 1 -o prof \\
        python bench/profile_kernels.py

Shapes (per rank at TP 8, batch 8, KV 2049): RMSNorm [8, 8192]; RoPE + KV write
for 8 query / 1 KV heads of 128; decode attention over 2049 cached tokens;
SiLU-gate [8, 2 x 3584]; decode GEMM [8, 8192] x [1280, 8192]^T; tcgen05 GEMM
[1024, 3584] x [8192, 3584]^T; fused residual + RMSNorm (one rank) [512, 8192].
"""

from __future__ import annotations

import os
import socket
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    from b200ar import CustomAllreduce
    from b200ar.ops.gemm import check_errors, linear
    from b200ar.ops.layers import RotaryTable, decode_attention, rmsnorm, rope_kv, silu_mul

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    comm = CustomAllreduce(device=dev, max_size=16 << 20)
    B, H, hq, hkv, d, L = 8, 8192, 8, 1, 128, 2049
    x = torch.randn(B, H, device=dev).to(torch.bfloat16)
    gamma = torch.ones(H, device=dev, dtype=torch.bfloat16)
    rot = RotaryTable(d, 4096, 500000.0, dev)
    qkv = torch.randn(B, (hq + 2 * hkv) * d, device=dev).to(torch.bfloat16)
    pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
    seq = torch.full((B,), L, dtype=torch.int32, device=dev)
    q = torch.empty(B, hq, d, device=dev, dtype=torch.bfloat16)
    kc = torch.randn(B, 4096, hkv, d, device=dev).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    gu = torch.randn(B, 2 * 3584, device=dev).to(torch.bfloat16)
    w_qkv = (0.02 * torch.randn(1280, H, device=dev)).to(torch.bfloat16)
    a_big = torch.randn(1024, 3584, device=dev).to(torch.bfloat16)
    w_big = (0.02 * torch.randn(8192, 3584, device=dev)).to(torch.bfloat16)
    xt = torch.randn(512, H, device=dev).to(torch.bfloat16)
    rt = torch.randn(512, H, device=dev).to(torch.bfloat16)

    def once():
        rmsnorm(x, gamma)
        rope_kv(qkv, pos, rot, q, kc, vc, hq, hkv)
        decode_attention(q, kc, vc, seq, hq, hkv)
        silu_mul(gu)
        linear(x, w_qkv)                 # split-K decode GEMM
        linear(a_big, w_big)             # persistent tcgen05 GEMM
        comm.all_reduce_residual_rmsnorm(xt, rt, torch.ones(H, device=dev, dtype=torch.bfloat16))

    once()  # warm-up pass
    torch.cuda.synchronize()
    once()  # profiled pass
    torch.cuda.synchronize()
    check_errors()
    comm.close()
    print("ok")


if __name__ == "__main__":
    main()
