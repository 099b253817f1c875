"""Fused tensor-parallel ops and their plain-PyTorch fp32 references."""

from __future__ import annotations

from typing import List, Tuple

import torch


def ref_ar_residual_rmsnorm(xs: List[torch.Tensor], residual: torch.Tensor, gamma: torch.Tensor,
                            eps: float = 1e-5) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 reference of ``all_reduce + residual add + RMSNorm`` given every
    rank's partial ``xs`` (summed in rank order). Returns (y, z) in the input
    dtype with z rounded once and the statistics taken on the rounded z, as the
    kernels do."""
    acc = xs[0].float()
    for t in xs[1:]:
        acc = acc + t.float()
    z = (acc + residual.float()).to(residual.dtype)
    zf = z.float()
    y = zf * torch.rsqrt(zf.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()
    return y.to(residual.dtype), z


def ar_residual_rmsnorm(comm, x, residual, gamma, eps: float = 1e-5, out=None, residual_out=None,
                        variant="auto"):
    """Functional form of ``CustomAllreduce.all_reduce_residual_rmsnorm``."""
    return comm.all_reduce_residual_rmsnorm(x, residual, gamma, eps, out=out, residual_out=residual_out,
                                            variant=variant)
