"""Decoder model kernels against plain-PyTorch fp32 references."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)


@pytest.mark.parametrize("rows,hidden", [(1, 8192), (33, 8192), (4, 4096), (7, 1024)])
def test_rmsnorm(rows, hidden):
    from b200ar.ops.layers import ref_rmsnorm, rmsnorm

    x = torch.randn(rows, hidden, device="cuda").to(torch.bfloat16)
    g = (1 + 0.01 * torch.randn(hidden, device="cuda")).to(torch.bfloat16)
    torch.testing.assert_close(rmsnorm(x, g).float(), ref_rmsnorm(x, g).float(), atol=2e-2, rtol=1e-2)


def test_rope_kv_writes_cache():
    from b200ar.ops.layers import RotaryTable, ref_rope, rope_kv

    b, hq, hkv, d, L = 3, 8, 1, 128, 64
    rot = RotaryTable(d, 4096, 500000.0, "cuda")
    qkv = torch.randn(b, (hq + 2 * hkv) * d, device="cuda").to(torch.bfloat16)
    pos = torch.tensor([0, 5, 63], dtype=torch.int32, device="cuda")
    q = torch.empty(b, hq, d, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(b, L, hkv, d, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    rope_kv(qkv, pos, rot, q, kc, vc, hq, hkv)
    x = qkv.view(b, hq + 2 * hkv, d)
    torch.testing.assert_close(q.float(), ref_rope(x[:, :hq], pos, rot), atol=2e-2, rtol=1e-2)
    for i in range(b):
        p = int(pos[i])
        torch.testing.assert_close(kc[i, p].float(), ref_rope(x[i:i + 1, hq:hq + hkv], pos[i:i + 1], rot)[0],
                                   atol=2e-2, rtol=1e-2)
        assert torch.equal(vc[i, p], x[i, hq + hkv:])


@pytest.mark.parametrize("impl", ["mma", "tc"])
@pytest.mark.parametrize("b,hq,hkv,L", [(1, 8, 1, 2049), (8, 8, 1, 2049), (4, 8, 2, 300), (2, 4, 4, 100),
                                        (3, 16, 1, 129), (64, 8, 1, 2049)])
def test_decode_attention(b, hq, hkv, L, impl):
    from b200ar.ops.gemm import check_errors
    from b200ar.ops.layers import decode_attention, ref_decode_attention

    q = torch.randn(b, hq, 128, device="cuda").to(torch.bfloat16)
    kc = torch.randn(b, L + 16, hkv, 128, device="cuda").to(torch.bfloat16)
    vc = torch.randn(b, L + 16, hkv, 128, device="cuda").to(torch.bfloat16)
    # Cache rows past each sequence hold NaN: a kernel must never let them reach the output.
    kc[:, L - 2:] = float("nan")
    vc[:, L - 2:] = float("nan")
    seq = torch.tensor([L - 2 - (i % 3) for i in range(b)], dtype=torch.int32, device="cuda")
    out = decode_attention(q, kc, vc, seq, hq, hkv, impl=impl)
    ref = ref_decode_attention(q, kc, vc, seq, hq, hkv)
    torch.cuda.synchronize()
    check_errors()
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


def test_silu_mul():
    from b200ar.ops.layers import ref_silu_mul, silu_mul

    gu = torch.randn(5, 2 * 3584, device="cuda").to(torch.bfloat16)
    torch.testing.assert_close(silu_mul(gu).float(), ref_silu_mul(gu).float(), atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("impl", ["mma", "tc"])
@pytest.mark.parametrize("splits", [1, 3, 64])
def test_decode_attention_merge_rearms(splits, impl):
    """The last split CTA merges the partials and re-arms its counter: repeated
    eager calls and CUDA-graph replays must keep matching the reference."""
    from b200ar.ops.layers import decode_attention, ref_decode_attention

    b, hq, hkv, L = 4, 8, 1, 1024 + 40
    q = torch.randn(b, hq, 128, device="cuda").to(torch.bfloat16)
    kc = torch.randn(b, L, hkv, 128, device="cuda").to(torch.bfloat16)
    vc = torch.randn(b, L, hkv, 128, device="cuda").to(torch.bfloat16)
    seq = torch.tensor([L, L - 7, 1, 0], dtype=torch.int32, device="cuda")
    out = torch.empty(b, hq * 128, dtype=torch.bfloat16, device="cuda")
    for _ in range(3):
        decode_attention(q, kc, vc, seq, hq, hkv, out=out, splits=splits, impl=impl)
    ref = ref_decode_attention(q, kc, vc, seq, hq, hkv)
    torch.testing.assert_close(out.float()[:3], ref[:3], atol=2e-2, rtol=2e-2)
    assert torch.equal(out[3], torch.zeros_like(out[3]))  # empty sequence -> zeros
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        decode_attention(q, kc, vc, seq, hq, hkv, out=out, splits=splits, impl=impl)
    for _ in range(3):
        q.copy_(torch.randn_like(q, dtype=torch.float32).to(torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        ref = ref_decode_attention(q, kc, vc, seq, hq, hkv)
        torch.testing.assert_close(out.float()[:3], ref[:3], atol=2e-2, rtol=2e-2)


def test_silu_mul_interleaved_groups():
    from b200ar.ops.layers import ref_silu_mul, silu_mul

    gu = torch.randn(5, 2 * 1024, device="cuda").to(torch.bfloat16)
    torch.testing.assert_close(silu_mul(gu, group=64).float(), ref_silu_mul(gu, group=64).float(), atol=2e-2,
                               rtol=1e-2)
