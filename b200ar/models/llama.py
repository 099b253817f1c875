"""Tensor-parallel Llama-3-70B-shaped decoder slice built on b200ar kernels.

Benchmark configuration: hidden 8192, 64 query / 8 KV heads of 128, RoPE
theta 500000, SwiGLU FFN 28672, RMSNorm eps 1e-5, 8 layers, random-init bf16
weights ~ N(0, 0.02), KV cache pre-filled with 2048 random tokens, decode at
batch 1 / 8 / 32 / 64 under CUDA graphs, two fused all-reduces per layer.

Per rank (tensor parallel over ``world`` GPUs) one decode step of a layer is

    q,kv = rope(h @ Wqkv^T); kv -> cache      column parallel, RoPE + cache write fused into the GEMM
    a    = attention(q, cache)                GQA decode attention kernel
    o    = a @ Wo^T                           row parallel, partial sums
    h, x = RMSNorm(all_reduce(o) + x)         fused all-reduce + residual + RMSNorm
    m    = silu(h @ Wg^T) * (h @ Wu^T)        column parallel, activation fused into the GEMM
    d    = m @ Wd^T                           row parallel, partial sums
    h, x = RMSNorm(all_reduce(d) + x)         fused, with the next layer's norm weights

The residual stream ``x`` is replicated on every rank, as in Megatron-style TP.
``Wgu`` stores the gate and up rows interleaved in groups of 64, so each
128-row block of the decode GEMM holds matching gate and up rows and its
epilogue can apply the activation.
``ReferenceDecoder`` computes the same step with plain PyTorch ops (cuBLAS,
NCCL all-reduce, PyTorch attention) as the comparison baseline.
"""

from __future__ import annotations

import dataclasses
import math
from typing import List, Optional

import torch
import torch.distributed as dist

from ..ops.gemm import linear, linear_rope_kv, linear_silu_gate
from ..ops.layers import RotaryTable, decode_attention, rmsnorm, split_gate_up


@dataclasses.dataclass
class LlamaConfig:
    hidden: int = 8192
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 28672
    layers: int = 8
    eps: float = 1e-5
    theta: float = 500000.0
    init_std: float = 0.02

    @staticmethod
    def llama3_70b_slice(layers: int = 8) -> "LlamaConfig":
        return LlamaConfig(layers=layers)


class TPLlamaDecoder:
    """One rank of the tensor-parallel decoder slice.

    Args:
        comm: ``CustomAllreduce`` of the TP group (world size 1 works too).
        cfg: model shape.
        batch: decode batch size (static: the step is graph-captured).
        max_len: KV cache capacity in tokens.
        seed: sharded weights are drawn from ``seed + 1000 * rank``; the
            replicated RMSNorm weights from one seed shared by all ranks.
    """

    def __init__(self, comm, cfg: LlamaConfig, batch: int, max_len: int, seed: int = 0):
        self.comm = comm
        self.cfg = cfg
        self.world = comm.world
        self.rank = comm.rank
        self.device = comm.device
        w = self.world
        if cfg.heads % w or cfg.intermediate % w:
            raise ValueError("heads and intermediate size must divide the TP world size")
        if (cfg.intermediate // w) % 64:
            raise ValueError("the per-rank intermediate size must be a multiple of 64 (gate/up interleave groups)")
        self.hq = cfg.heads // w
        self.hkv = max(1, cfg.kv_heads // w)
        self.inter = cfg.intermediate // w
        self.batch = batch
        self.max_len = max_len
        d, H = cfg.head_dim, cfg.hidden
        # Sharded weights differ per rank; the RMSNorm weights are replicated
        # (like the residual stream), so every rank draws them from one seed.
        g = torch.Generator(device=self.device).manual_seed(seed + 1000 * self.rank)
        g_rep = torch.Generator(device=self.device).manual_seed(seed + 999_983)

        def rnd(*shape):
            return (cfg.init_std * torch.randn(*shape, generator=g, device=self.device)).to(torch.bfloat16)

        def gamma():
            return (1 + 0.01 * torch.randn(H, generator=g_rep, device=self.device)).to(torch.bfloat16)

        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "wqkv": rnd((self.hq + 2 * self.hkv) * d, H),
                "wo": rnd(H, self.hq * d),
                "wgu": rnd(2 * self.inter, H),
                "wd": rnd(H, self.inter),
                "g_attn": gamma(),
                "g_mlp": gamma(),
            })
        self.g_final = gamma()
        self.rot = RotaryTable(d, max_len, cfg.theta, self.device)
        self.k_cache = [torch.zeros(batch, max_len, self.hkv, d, dtype=torch.bfloat16, device=self.device)
                        for _ in range(cfg.layers)]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        # Static step buffers (graph capture needs fixed addresses).
        B = batch
        self.x = torch.zeros(B, H, dtype=torch.bfloat16, device=self.device)      # residual stream
        self.h = torch.zeros(B, H, dtype=torch.bfloat16, device=self.device)      # normed activations
        self.pos = torch.zeros(B, dtype=torch.int32, device=self.device)
        self.seq_len = torch.ones(B, dtype=torch.int32, device=self.device)
        self.qkv = torch.empty(B, (self.hq + 2 * self.hkv) * d, dtype=torch.bfloat16, device=self.device)
        self.q = torch.empty(B, self.hq, d, dtype=torch.bfloat16, device=self.device)
        self.attn = torch.empty(B, self.hq * d, dtype=torch.bfloat16, device=self.device)
        self.part = torch.empty(B, H, dtype=torch.bfloat16, device=self.device)
        self.gu = torch.empty(B, 2 * self.inter, dtype=torch.bfloat16, device=self.device)
        self.act = torch.empty(B, self.inter, dtype=torch.bfloat16, device=self.device)
        self.out = torch.empty(B, H, dtype=torch.bfloat16, device=self.device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    # ---------------------------------------------------------------- state
    def prefill_random(self, context: int, seed: int = 1) -> None:
        """Fills the first ``context`` KV positions with random values (same on
        all ranks' shards by seed) and sets the next decode position."""
        g = torch.Generator(device=self.device).manual_seed(seed + 7 * self.rank)
        for k, v in zip(self.k_cache, self.v_cache):
            k[:, :context].normal_(generator=g)
            v[:, :context].normal_(generator=g)
        self.pos.fill_(context)
        self.seq_len.fill_(context + 1)

    def set_input(self, x: torch.Tensor) -> None:
        self.x.copy_(x)

    # ---------------------------------------------------------------- step
    def _layer(self, i: int, first: bool) -> None:
        L = self.layers[i]
        cfg = self.cfg
        if first:
            rmsnorm(self.x, L["g_attn"], cfg.eps, out=self.h)
        linear_rope_kv(self.h, L["wqkv"], self.pos, self.rot, self.q, self.k_cache[i], self.v_cache[i], self.hq,
                       self.hkv, scratch=self.qkv)
        decode_attention(self.q, self.k_cache[i], self.v_cache[i], self.seq_len, self.hq, self.hkv, out=self.attn)
        linear(self.attn, L["wo"], out=self.part)
        self.comm.all_reduce_residual_rmsnorm(self.part, self.x, L["g_mlp"], cfg.eps, out=self.h,
                                              residual_out=self.x)
        linear_silu_gate(self.h, L["wgu"], out=self.act, scratch=self.gu)
        linear(self.act, L["wd"], out=self.part)
        nxt = self.layers[i + 1]["g_attn"] if i + 1 < len(self.layers) else self.g_final
        self.comm.all_reduce_residual_rmsnorm(self.part, self.x, nxt, cfg.eps, out=self.h, residual_out=self.x)

    def forward_step(self) -> torch.Tensor:
        """One decode step for every sequence of the batch; returns the final
        normalised hidden state [B, hidden] (``self.h``). Advances positions."""
        for i in range(len(self.layers)):
            self._layer(i, first=(i == 0))
        self.pos.add_(1)
        self.seq_len.add_(1)
        return self.h

    def capture(self) -> torch.cuda.CUDAGraph:
        """Captures ``forward_step`` into a CUDA graph (after one eager warm-up
        step; the warm-up advances positions by one, which is undone)."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        x0 = self.x.clone()
        with torch.cuda.stream(s):
            self.forward_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.pos.sub_(1)
        self.seq_len.sub_(1)
        self.x.copy_(x0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward_step()
        self.graph = g
        return g

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.h


class ReferenceDecoder:
    """The same decoder step with plain PyTorch ops: cuBLAS matmuls, NCCL
    all-reduce, PyTorch RMSNorm/RoPE/attention. Shares weights, caches and
    buffers with a ``TPLlamaDecoder`` so both compute the same function."""

    def __init__(self, model: TPLlamaDecoder, group=None, allreduce=None):
        self.m = model
        self.group = group
        self.allreduce = allreduce  # callable(tensor) -> None (in place); default NCCL
        self.graph = None

    def _ar(self, t):
        if self.m.world == 1:
            return
        if self.allreduce is not None:
            self.allreduce(t)
        else:
            dist.all_reduce(t, group=self.group)

    @staticmethod
    def _norm(x, g, eps):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * g.float()).to(torch.bfloat16)

    def _rope(self, t):  # t [B, H, d]
        m = self.m
        half = t.shape[-1] // 2
        c = m.rot.cos[m.pos.long()][:, None, :]
        s = m.rot.sin[m.pos.long()][:, None, :]
        x0, x1 = t[..., :half].float(), t[..., half:].float()
        return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1).to(torch.bfloat16)

    def forward_step(self):
        m = self.m
        cfg = m.cfg
        B, d = m.batch, cfg.head_dim
        idx = m.pos.long()
        ar = torch.arange(B, device=m.device)
        for i, L in enumerate(m.layers):
            if i == 0:
                m.h.copy_(self._norm(m.x, L["g_attn"], cfg.eps))
            qkv = (m.h @ L["wqkv"].t()).view(B, m.hq + 2 * m.hkv, d)
            q = self._rope(qkv[:, :m.hq])
            k = self._rope(qkv[:, m.hq:m.hq + m.hkv])
            m.k_cache[i][ar, idx] = k
            m.v_cache[i][ar, idx] = qkv[:, m.hq + m.hkv:]
            # Attention over the first seq_len positions (the same length for the whole batch here).
            capturing = m.device.type == "cuda" and torch.cuda.is_current_stream_capturing()
            n = self._cap_len if capturing else int(m.seq_len[0])
            kk = m.k_cache[i][:, :n].transpose(1, 2)  # [B, hkv, n, d]
            vv = m.v_cache[i][:, :n].transpose(1, 2)
            a = torch.nn.functional.scaled_dot_product_attention(q.unsqueeze(2), kk, vv, enable_gqa=True)
            part = a.reshape(B, m.hq * d) @ L["wo"].t()
            self._ar(part)
            m.x.copy_((part.float() + m.x.float()).to(torch.bfloat16))
            m.h.copy_(self._norm(m.x, L["g_mlp"], cfg.eps))
            gu = m.h @ L["wgu"].t()
            g, u = split_gate_up(gu, 64)
            act = (torch.nn.functional.silu(g.float()) * u.float()).to(torch.bfloat16)
            part = act @ L["wd"].t()
            self._ar(part)
            m.x.copy_((part.float() + m.x.float()).to(torch.bfloat16))
            nxt = m.layers[i + 1]["g_attn"] if i + 1 < len(m.layers) else m.g_final
            m.h.copy_(self._norm(m.x, nxt, cfg.eps))
        m.pos.add_(1)
        m.seq_len.add_(1)
        return m.h

    def capture(self):
        """Graph capture; the attention length is fixed at capture time (a
        static-shape restriction of the PyTorch baseline)."""
        m = self.m
        s = torch.cuda.Stream(device=m.device)
        s.wait_stream(torch.cuda.current_stream(m.device))
        x0 = m.x.clone()
        with torch.cuda.stream(s):
            self.forward_step()
        torch.cuda.current_stream(m.device).wait_stream(s)
        torch.cuda.synchronize(m.device)
        m.pos.sub_(1)
        m.seq_len.sub_(1)
        m.x.copy_(x0)
        self._cap_len = int(m.seq_len[0])
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward_step()
        self.graph = g
        return g
