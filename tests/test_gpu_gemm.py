"""tcgen05 GEMM against a PyTorch fp32 reference of the same op."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)


@pytest.mark.parametrize(
    "m,n,k",
    [(128, 256, 64), (16, 8192, 3584), (128, 8192, 3584), (1024, 8192, 3584), (1, 512, 128), (200, 264, 72),
     (4096, 1024, 8192)],
)
def test_gemm_matches_fp32(m, n, k):
    from b200ar.ops.gemm import check_errors, linear

    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, generator=g, device="cuda")).to(torch.bfloat16)
    out = linear(a, w)
    out1 = linear(a, w, pair=False)  # single-CTA tiles (the fused GEMM + all-reduce main loop)
    torch.cuda.synchronize()
    check_errors()
    ref = a.float() @ w.float().t()
    assert (out1.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-2
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-2 * scale + 1e-2, (err, scale)


def test_gemm_repeated_and_capped_grid():
    from b200ar.ops.gemm import check_errors, linear

    a = torch.randn(512, 1024, device="cuda").to(torch.bfloat16)
    w = torch.randn(2048, 1024, device="cuda").to(torch.bfloat16)
    ref = (a.float() @ w.float().t()).to(torch.bfloat16)
    for ctas in (1, 3, 0):
        out = linear(a, w, max_ctas=ctas)
        torch.cuda.synchronize()
        check_errors()
        torch.testing.assert_close(out.float(), ref.float(), atol=0.5, rtol=2e-2)


@pytest.mark.parametrize("m", [1, 8, 16, 17, 32, 64, 100, 128])
@pytest.mark.parametrize("n,k", [(1280, 8192), (8192, 1024), (7168, 8192), (8192, 3584), (264, 136)])
def test_skinny_gemm_matches_fp32(m, n, k):
    from b200ar.ops.gemm import check_errors, linear

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, generator=g, device="cuda")).to(torch.bfloat16)
    for _ in range(2):  # the split-K counters must be reset by the first call
        out = linear(a, w, skinny=True)
        torch.cuda.synchronize()
        check_errors()
        ref = a.float() @ w.float().t()
        err = (out.float() - ref).abs().max().item()
        assert err <= 1e-2 * ref.abs().max().item() + 1e-2, (m, n, k, err)


@pytest.mark.parametrize("m,inter,k", [(1, 3584, 8192), (8, 3584, 8192), (64, 512, 1024), (128, 1024, 256),
                                       (200, 512, 256)])
def test_linear_silu_gate_fused_epilogue(m, inter, k):
    """The fused SiLU-gate epilogue equals the GEMM followed by the activation
    kernel bit for bit (same split order, same bf16 rounding of gate and up),
    and both match an fp32 reference."""
    from b200ar.ops.gemm import check_errors, linear, linear_silu_gate
    from b200ar.ops.layers import ref_silu_mul, silu_mul

    g = torch.Generator(device="cuda").manual_seed(m + inter + k)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(2 * inter, k, generator=g, device="cuda")).to(torch.bfloat16)
    fused = linear_silu_gate(x, w)
    two_step = silu_mul(linear(x, w, skinny=m <= 128), group=64)  # the product the fused path runs
    torch.cuda.synchronize()
    check_errors()
    assert torch.equal(fused, two_step)
    ref = ref_silu_mul((x.float() @ w.float().t()).to(torch.bfloat16), group=64)
    torch.testing.assert_close(fused.float(), ref.float(), atol=2e-2, rtol=2e-2)
    for _ in range(3):  # repeated calls re-arm the split-K counters
        again = linear_silu_gate(x, w)
    torch.cuda.synchronize()
    assert torch.equal(again, fused)


@pytest.mark.parametrize("b,hq,hkv", [(1, 8, 1), (8, 8, 1), (3, 4, 2), (64, 8, 1)])
def test_linear_rope_kv_fused_epilogue(b, hq, hkv):
    """The QKV GEMM with RoPE + KV write in its epilogue matches the GEMM
    followed by the RoPE kernel (v bit for bit; q and k to one bf16 ulp)."""
    from b200ar.ops.gemm import check_errors, linear, linear_rope_kv
    from b200ar.ops.layers import RotaryTable, rope_kv

    H, L = 1024, 96
    g = torch.Generator(device="cuda").manual_seed(b * 31 + hq + hkv)
    x = torch.randn(b, H, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.05 * torch.randn((hq + 2 * hkv) * 128, H, generator=g, device="cuda")).to(torch.bfloat16)
    pos = torch.randint(0, L, (b,), generator=g, device="cuda", dtype=torch.int32)
    rot = RotaryTable(128, L, 500000.0, "cuda")
    q1 = torch.empty(b, hq, 128, dtype=torch.bfloat16, device="cuda")
    k1 = torch.zeros(b, L, hkv, 128, dtype=torch.bfloat16, device="cuda")
    v1 = torch.zeros_like(k1)
    q2, k2, v2 = torch.empty_like(q1), torch.zeros_like(k1), torch.zeros_like(v1)
    for _ in range(2):  # the second call re-uses the re-armed counters
        linear_rope_kv(x, w, pos, rot, q1, k1, v1, hq, hkv)
    rope_kv(linear(x, w, skinny=True), pos, rot, q2, k2, v2, hq, hkv)
    torch.cuda.synchronize()
    check_errors()
    assert torch.equal(v1, v2)
    torch.testing.assert_close(q1.float(), q2.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(k1.float(), k2.float(), atol=2e-2, rtol=1e-2)
    assert torch.count_nonzero(k1) == torch.count_nonzero(k2)  # only positions `pos` were written


@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (300, 520, 200), (1024, 8192, 3584), (8192, 1024, 1024),
                                   (4096, 4096, 512)])
def test_gemm_cta_pair_matches_fp32(m, n, k):
    """The cta_group::2 kernel (256 x 256 tiles over two SMs) against fp32."""
    from b200ar.ops.gemm import check_errors, linear

    g = torch.Generator(device="cuda").manual_seed(m + 3 * n + k)
    a = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, generator=g, device="cuda")).to(torch.bfloat16)
    for pairs in (0, 1, 3):  # persistent loop over tiles when the grid is capped
        out = linear(a, w, skinny=False, pair=True, max_ctas=2 * pairs)
        torch.cuda.synchronize()
        check_errors()
        ref = a.float() @ w.float().t()
        err = (out.float() - ref).abs().max().item()
        scale = ref.abs().max().item()
        assert err <= 1e-2 * scale + 1e-2, (pairs, err, scale)
