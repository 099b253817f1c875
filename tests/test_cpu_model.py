"""The tensor-parallel decoder slice on the CPU backend (gloo ranks + shared
memory): the TP step (sharded weights, fused all-reduce + residual + RMSNorm,
row/column-parallel linears) against the plain-PyTorch reference step on the
same weights and caches, and the fused linear collectives against fp32
oracles. Exercises the sharding and data flow without a GPU."""

import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks


def _tp_decoder(rank, world):
    from b200ar import CustomAllreduce
    from b200ar.models.llama import LlamaConfig, ReferenceDecoder, TPLlamaDecoder

    comm = CustomAllreduce(device="cpu", max_size=4 << 20)
    cfg = LlamaConfig(hidden=256, heads=4 * world, kv_heads=world, head_dim=128, intermediate=512 * world,
                      layers=2)
    B, ctx = 3, 20
    m = TPLlamaDecoder(comm, cfg, batch=B, max_len=64, seed=3)
    m.prefill_random(ctx)
    x0 = torch.randn(B, cfg.hidden, generator=torch.Generator().manual_seed(11)).to(torch.bfloat16)
    kc = [k.clone() for k in m.k_cache]
    vc = [v.clone() for v in m.v_cache]
    m.set_input(x0)
    ours = m.forward_step().clone()
    assert int(m.pos[0]) == ctx + 1 and int(m.seq_len[0]) == ctx + 2
    # The residual stream and the normalised output are replicated: every rank
    # holds bitwise the same values (sums run in rank order everywhere).
    outs = [None] * world
    dist.all_gather_object(outs, ours)
    assert all(torch.equal(o, outs[0]) for o in outs)
    # Same weights, caches and input through the plain-PyTorch step.
    for k, k0 in zip(m.k_cache, kc):
        k.copy_(k0)
    for v, v0 in zip(m.v_cache, vc):
        v.copy_(v0)
    m.pos.fill_(ctx)
    m.seq_len.fill_(ctx + 1)
    m.set_input(x0)
    ref = ReferenceDecoder(m, allreduce=lambda t: comm.all_reduce(t, out=t)).forward_step().clone()
    err = (ours.float() - ref.float()).abs().max().item()
    assert err < 0.1, err
    comm.close()


@pytest.mark.parametrize("world", [1, 2])
def test_tp_decoder_matches_reference_step(world):
    run_ranks(_tp_decoder, world)


def _linear_collectives(rank, world):
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=4 << 20)
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(6, 64, generator=g).to(torch.bfloat16)
    w = (0.1 * torch.randn(48, 64, generator=g)).to(torch.bfloat16)
    xs, ws = [None] * world, [None] * world
    dist.all_gather_object(xs, x)
    dist.all_gather_object(ws, w)
    # Row parallel: sum over ranks of x_r @ w_r^T.
    ref = sum(a.float() @ b.float().t() for a, b in zip(xs, ws))
    out = comm.linear_all_reduce(x, w)
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)
    # Column parallel on sequence-sharded rows: concat_r(x_r) @ w^T.
    full = comm.all_gather_linear(x, w)
    torch.testing.assert_close(full.float(), torch.cat(xs).float() @ w.float().t(), atol=3e-2, rtol=2e-2)
    comm.close()


@pytest.mark.parametrize("world", [1, 2])
def test_linear_collectives_cpu(world):
    run_ranks(_linear_collectives, world)


def _step_bytes(rank, world):
    import importlib.util
    import os

    from b200ar import CustomAllreduce
    from b200ar.models.llama import LlamaConfig, TPLlamaDecoder

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("decoder_bench", os.path.join(root, "bench", "decoder_bench.py"))
    db = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(db)
    comm = CustomAllreduce(device="cpu", max_size=1 << 20)
    cfg = LlamaConfig(hidden=256, heads=4, kv_heads=1, head_dim=128, intermediate=512, layers=2)
    m = TPLlamaDecoder(comm, cfg, batch=2, max_len=32)
    m.prefill_random(10)
    H, d = 256, 128
    weights = 2 * 2 * ((4 + 2) * d * H + H * 4 * d + 2 * 512 * H + H * 512 + 2 * H)  # 2 layers, bf16
    kv = 11 * (2 * 1 * d * 2 * 2) * 2  # seq_len 11, k and v, 2 layers, batch 2
    assert db.step_bytes(m) == weights + kv
    comm.close()


def test_decoder_bench_step_bytes():
    run_ranks(_step_bytes, 1)
