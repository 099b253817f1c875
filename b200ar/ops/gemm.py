"""bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).

``linear(x, w)`` computes ``x @ w.T`` for ``x [M, K]`` and ``w [N, K]`` (the
``nn.Linear`` weight layout) with the hand-written sm_100a kernel in
``csrc/gemm``; fp32 accumulation, bf16 output.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from .._native import _C

_ERR: Dict[int, torch.Tensor] = {}


def error_word(device) -> torch.Tensor:
    """Per-device int32 that a kernel sets when one of its bounded waits expires."""
    idx = torch.device(device).index or 0
    if idx not in _ERR:
        _ERR[idx] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
    return _ERR[idx]


def check_errors(device=None) -> None:
    """Raises if a GEMM reported an expired wait (synchronises the device)."""
    for idx, t in _ERR.items():
        if device is not None and idx != (torch.device(device).index or 0):
            continue
        v = int(t.item())
        if v:
            t.zero_()
            raise RuntimeError(f"tcgen05 GEMM on cuda:{idx} reported error {v} (a bounded wait expired)")


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None, max_ctas: int = 0) -> torch.Tensor:
    """``x @ w.T`` (bf16). ``x``: [..., K]; ``w``: [N, K]."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x2.shape[0], w.shape[0], dtype=torch.bfloat16, device=x.device)
    _C.gemm_bf16(x2, w, out.view(x2.shape[0], w.shape[0]), error_word(x.device), max_ctas)
    return out.view(*shp[:-1], w.shape[0])
