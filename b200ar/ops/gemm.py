"""bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).

``linear(x, w)`` computes ``x @ w.T`` for ``x [M, K]`` and ``w [N, K]`` (the
``nn.Linear`` weight layout) with the hand-written sm_100a kernel in
``csrc/gemm``; fp32 accumulation, bf16 output. CPU tensors (the plumbing
backend) use the fp32 reference product.
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


_SKINNY: Dict[int, dict] = {}

# Plain products up to this many rows run the split-K decode kernel; wider
# ones the CTA-pair kernel, which was measured faster from 128 rows
# (18.4 vs 25.6 us at 128 x 8192 x 1024, 32.8 vs 35.0 us at 128 x 8192 x 3584).
# The fused SiLU-gate and RoPE + KV epilogues keep the decode kernel up to 128 rows.
SKINNY_MAX_ROWS = 64


def _skinny_workspace(device, splits: int, m: int, n: int):
    """Per-device split-K scratch: fp32 partials and zeroed arrival counters
    (reused by every decode GEMM on that device; calls are stream-ordered)."""
    idx = torch.device(device).index or 0
    ws = _SKINNY.setdefault(idx, {})
    need = splits * m * n
    if ws.get("partials") is None or ws["partials"].numel() < need:
        ws["partials"] = torch.empty(max(need, 1 << 20), dtype=torch.float32, device=device)
    blocks = (n + 127) // 128
    if ws.get("counters") is None or ws["counters"].numel() < blocks:
        ws["counters"] = torch.zeros(max(blocks, 1024), dtype=torch.int32, device=device)
    if "sms" not in ws:
        ws["sms"] = torch.cuda.get_device_properties(device).multi_processor_count
    return ws


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None, max_ctas: int = 0,
           skinny: Optional[bool] = None, pair: bool = True) -> torch.Tensor:
    """``x @ w.T`` (bf16). ``x``: [..., K]; ``w``: [N, K]. Up to
    ``SKINNY_MAX_ROWS`` rows (or up to 128 with ``skinny=True``) use the split-K
    decode kernel; other shapes run on CTA pairs (tcgen05 cta_group::2,
    256 x 256 tiles; 10-14 % faster than single-CTA 128 x 256 tiles on B200),
    or on single CTAs with ``pair=False``.
    ``max_ctas`` caps the persistent grid (rounded down to whole pairs)."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    m, n = x2.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    out2 = out.view(m, n)
    if x.device.type == "cpu":  # plumbing backend: fp32 reference math, never a CUDA fallback
        out2.copy_((x2.float() @ w.float().t()).to(out2.dtype))
        return out.view(*shp[:-1], n)
    if skinny is None:
        skinny = m <= SKINNY_MAX_ROWS
    if skinny:
        ws = _skinny_workspace(x.device, 1, m, n)
        splits = _C.skinny_splits(n, x2.shape[1], ws["sms"])
        ws = _skinny_workspace(x.device, splits, m, n)
        _C.gemm_skinny(x2, w, out2, ws["partials"], ws["counters"], error_word(x.device), splits)
    elif pair:
        _C.gemm_bf16_2sm(x2, w, out2, error_word(x.device), max(1, max_ctas // 2) if max_ctas > 0 else 0)
    else:
        _C.gemm_bf16(x2, w, out2, error_word(x.device), max_ctas)
    return out.view(*shp[:-1], n)


def linear_silu_gate(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                     scratch: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(x @ Wg^T) * (x @ Wu^T)`` where the rows of ``w`` [2 I, K] hold the
    gate and up projections interleaved in groups of 64 (rows 128 j .. 128 j +
    63 gate, the next 64 the matching up rows). Decode batches (rows <= 128)
    run one tcgen05 GEMM whose split-K reduction applies the activation; other
    shapes run the GEMM into ``scratch`` [rows, 2 I] and the activation kernel."""
    from .layers import silu_mul

    x2 = x.reshape(-1, x.shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    m, n = x2.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(m, n // 2, dtype=torch.bfloat16, device=x.device)
    if x.device.type == "cpu" or m > 128 or n % 128:
        gu = linear(x2, w, out=scratch)
        return silu_mul(gu.view(m, n), out=out, group=64)
    ws = _skinny_workspace(x.device, 1, m, n)
    splits = _C.skinny_splits(n, x2.shape[1], ws["sms"])
    ws = _skinny_workspace(x.device, splits, m, n)
    _C.gemm_skinny(x2, w, out.view(m, n // 2), ws["partials"], ws["counters"], error_word(x.device), splits, 1)
    return out


def linear_rope_kv(x: torch.Tensor, wqkv: torch.Tensor, pos: torch.Tensor, rot, q_out: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, hq: int, hkv: int,
                   scratch: Optional[torch.Tensor] = None) -> None:
    """QKV projection with RoPE and the KV-cache write: ``qkv = x @ Wqkv^T``
    (heads of 128 rows, [q | k | v]); q and k rotated at ``pos`` (rotate-half),
    q to ``q_out`` [B, hq, 128], k and v into the caches [B, L, hkv, 128] at
    ``pos``. Decode batches (rows <= 128, head_dim 128) run one tcgen05 GEMM
    whose split-K reduction does the rotation and the cache write; other
    shapes run the GEMM into ``scratch`` and the RoPE kernel."""
    from .layers import rope_kv

    m, n = x.shape[0], wqkv.shape[0]
    if x.device.type == "cpu" or m > 128 or rot.head_dim != 128 or n != (hq + 2 * hkv) * 128:
        qkv = linear(x, wqkv, out=scratch)
        rope_kv(qkv, pos, rot, q_out, k_cache, v_cache, hq, hkv)
        return
    x2 = x if x.is_contiguous() else x.contiguous()
    ws = _skinny_workspace(x.device, 1, m, n)
    splits = _C.skinny_splits(n, x2.shape[1], ws["sms"])
    ws = _skinny_workspace(x.device, splits, m, n)
    _C.gemm_skinny_rope_kv(x2, wqkv, pos, rot.cos, rot.sin, q_out, k_cache, v_cache, ws["partials"],
                           ws["counters"], error_word(x.device), splits, hq, hkv)
