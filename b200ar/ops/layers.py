"""Decoder layer ops on the hand-written sm_100a kernels (``csrc/model``),
each with a plain-PyTorch fp32 reference used by the tests.

* ``rmsnorm``            y = x * rsqrt(mean(x^2) + eps) * gamma
* ``RotaryTable``        cos/sin tables for RoPE (theta, head_dim, max positions)
* ``rope_kv``            rotate q and k (rotate-half convention), write k and v into the KV cache
* ``decode_attention``   GQA decode attention over the KV cache (split-KV, online softmax)
* ``silu_mul``           silu(gate) * up

CUDA tensors always run the sm_100a kernels. CPU tensors (the gloo/shared-memory
plumbing backend, used to test tensor-parallel logic without a GPU) run the
fp32 reference math of each op; no CUDA call falls back to it.
"""

from __future__ import annotations

import math
from typing import Dict, Tuple

import torch

from .._native import _C


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5, out=None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    if x.device.type == "cpu":
        out.copy_(ref_rmsnorm(x, gamma, eps))
        return out
    if torch.compiler.is_compiling():  # traced: the dispatcher op of the same kernel
        torch.ops.b200ar.rmsnorm(x.contiguous(), gamma, float(eps), out)
        return out
    _C.rmsnorm(x.contiguous(), gamma, out, float(eps))
    return out


def ref_rmsnorm(x, gamma, eps=1e-5):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()).to(x.dtype)


class RotaryTable:
    """cos/sin of position * theta^(-2i/d) for i < d/2, fp32 on the device."""

    def __init__(self, head_dim: int, max_pos: int, theta: float, device):
        inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
        ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos = ang.cos().float().to(device).contiguous()
        self.sin = ang.sin().float().to(device).contiguous()
        self.head_dim = head_dim


def rope_kv(qkv, pos, rot: RotaryTable, q_out, k_cache, v_cache, hq: int, hkv: int) -> None:
    """qkv [B, (hq + 2 hkv) * d] -> q_out [B, hq, d]; k, v into caches [B, L, hkv, d] at ``pos``."""
    if qkv.device.type == "cpu":
        b, d = qkv.shape[0], rot.head_dim
        x = qkv.view(b, hq + 2 * hkv, d)
        q_out.copy_(ref_rope(x[:, :hq], pos, rot).to(q_out.dtype))
        rows, idx = torch.arange(b), pos.long()
        k_cache[rows, idx] = ref_rope(x[:, hq:hq + hkv], pos, rot).to(k_cache.dtype)
        v_cache[rows, idx] = x[:, hq + hkv:].to(v_cache.dtype)
        return
    _C.rope_kv(qkv, pos, rot.cos, rot.sin, q_out, k_cache, v_cache, hq, hkv, rot.head_dim)


def ref_rope(x, pos, rot: RotaryTable):
    """x [B, H, d] fp32 reference of the rotate-half rotation."""
    half = x.shape[-1] // 2
    c = rot.cos[pos.long()][:, None, :]
    s = rot.sin[pos.long()][:, None, :]
    x0, x1 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1)


# Per (device, partial count, counter count): fp32 partial outputs, fp32
# (max, sum) pairs and the int32 per-(batch, KV head) arrival counters, which
# start at zero and are re-armed by the kernel itself.
_ATTN_WS: Dict[Tuple[int, int, int], Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}


def decode_attention(q, k_cache, v_cache, seq_len, hq: int, hkv: int, out=None, splits: int = 0,
                     impl: str = "tc"):
    """q [B, hq, 128]; caches [B, L, hkv, 128]; seq_len int32 [B] -> out [B, hq * 128].

    ``impl`` "tc" (default): tcgen05 tensor cores with TMA-fed K/V; "mma": the
    earlier mma.sync kernel, kept as the comparison point of
    ``bench/attention_bench.py``."""
    b = q.shape[0]
    if out is None:
        out = torch.empty(b, hq * 128, dtype=q.dtype, device=q.device)
    if q.device.type == "cpu":
        out.copy_(ref_decode_attention(q, k_cache, v_cache, seq_len, hq, hkv).to(out.dtype))
        return out
    tc = impl == "tc"
    if splits <= 0:
        splits = (_C.attention_tc_splits if tc else _C.attention_splits)(b, hkv, k_cache.shape[1])
    key = (q.device.index or 0, b * hq * splits, b * hkv)
    if key not in _ATTN_WS:
        _ATTN_WS[key] = (torch.empty(b * hq * splits * 128, dtype=torch.float32, device=q.device),
                         torch.empty(b * hq * splits * 2, dtype=torch.float32, device=q.device),
                         torch.zeros(b * hkv, dtype=torch.int32, device=q.device))
    acc, ml, cnt = _ATTN_WS[key]
    if tc:
        from .gemm import error_word

        _C.decode_attention_tc(q, k_cache, v_cache, seq_len, out, acc, ml, cnt, error_word(q.device), hq, hkv, splits,
                               1.0 / math.sqrt(128))
    else:
        _C.decode_attention(q, k_cache, v_cache, seq_len, out, acc, ml, cnt, hq, hkv, splits, 1.0 / math.sqrt(128))
    return out


def ref_decode_attention(q, k_cache, v_cache, seq_len, hq: int, hkv: int):
    b = q.shape[0]
    g = hq // hkv
    out = torch.empty(b, hq, 128, dtype=torch.float32, device=q.device)
    for i in range(b):
        n = int(seq_len[i])
        k = k_cache[i, :n].float().repeat_interleave(g, dim=1)  # [n, hq, d]
        v = v_cache[i, :n].float().repeat_interleave(g, dim=1)
        sc = torch.einsum("hd,nhd->hn", q[i].float(), k) / math.sqrt(128)
        p = torch.softmax(sc, dim=-1)
        out[i] = torch.einsum("hn,nhd->hd", p, v)
    return out.reshape(b, hq * 128)


def silu_mul(gate_up, out=None, group: int = 0):
    """silu(gate) * up. ``group`` 0: ``gate_up`` is [gate | up]; ``group`` g:
    gate and up columns alternate in groups of g (the layout whose gate-up
    GEMM can fuse the activation, see ``b200ar.ops.gemm.linear_silu_gate``)."""
    rows, two_i = gate_up.shape
    if out is None:
        out = torch.empty(rows, two_i // 2, dtype=gate_up.dtype, device=gate_up.device)
    if gate_up.device.type == "cpu":
        out.copy_(ref_silu_mul(gate_up, group))
        return out
    if torch.compiler.is_compiling():
        torch.ops.b200ar.silu_mul(gate_up, out, group)
        return out
    _C.silu_mul(gate_up, out, group)
    return out


def split_gate_up(gate_up, group: int = 0):
    """(gate, up) views of a gate-up product in either layout of ``silu_mul``."""
    rows, two_i = gate_up.shape
    if group == 0:
        return gate_up.chunk(2, dim=-1)
    g = gate_up.view(rows, two_i // (2 * group), 2, group)
    return g[:, :, 0].reshape(rows, -1), g[:, :, 1].reshape(rows, -1)


def ref_silu_mul(gate_up, group: int = 0):
    g, u = split_gate_up(gate_up.float(), group)
    return (torch.nn.functional.silu(g) * u).to(gate_up.dtype)
