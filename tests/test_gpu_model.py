"""TP Llama decoder slice: b200ar kernels vs the plain-PyTorch reference step."""

import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)


def _compare(rank, world):
    from b200ar import CustomAllreduce
    from b200ar.models.llama import LlamaConfig, ReferenceDecoder, TPLlamaDecoder

    gloo = dist.new_group(backend="gloo")
    comm = CustomAllreduce(group=gloo, device=torch.device("cuda", rank),
                           nccl_group=dist.group.WORLD if world > 1 else None, max_size=8 << 20)
    cfg = LlamaConfig(hidden=1024, heads=8 * world, kv_heads=world, head_dim=128, intermediate=2048 * world,
                      layers=2)
    B = 4
    m = TPLlamaDecoder(comm, cfg, batch=B, max_len=256, seed=3)
    m.prefill_random(100)
    x0 = (torch.randn(B, cfg.hidden, generator=torch.Generator(device="cuda").manual_seed(11), device="cuda")
          ).to(torch.bfloat16)
    kc = [k.clone() for k in m.k_cache]
    vc = [v.clone() for v in m.v_cache]
    m.set_input(x0)
    ours = m.forward_step().clone()
    # Reset state and run the reference on the same weights/caches.
    for k, k0 in zip(m.k_cache, kc):
        k.copy_(k0)
    for v, v0 in zip(m.v_cache, vc):
        v.copy_(v0)
    m.pos.fill_(100)
    m.seq_len.fill_(101)
    m.set_input(x0)
    ref = ReferenceDecoder(m).forward_step().clone()
    torch.cuda.synchronize()
    err = (ours.float() - ref.float()).abs().max().item()
    assert err < 0.1, err
    # Graph-captured steps advance positions and keep producing finite output.
    m.capture()
    for _ in range(3):
        h = m.replay()
    torch.cuda.synchronize()
    assert bool(torch.isfinite(h.float()).all())
    comm.check()
    comm.close()


def test_decoder_world1():
    run_ranks(_compare, 1, backend="nccl")


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_decoder_world2():
    run_ranks(_compare, 2, backend="nccl")
