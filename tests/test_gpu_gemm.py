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
    torch.cuda.synchronize()
    check_errors()
    ref = a.float() @ w.float().t()
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
    two_step = silu_mul(linear(x, w), group=64)
    torch.cuda.synchronize()
    check_errors()
    assert torch.equal(fused, two_step)
    ref = ref_silu_mul((x.float() @ w.float().t()).to(torch.bfloat16), group=64)
    torch.testing.assert_close(fused.float(), ref.float(), atol=2e-2, rtol=2e-2)
    for _ in range(3):  # repeated calls re-arm the split-K counters
        again = linear_silu_gate(x, w)
    torch.cuda.synchronize()
    assert torch.equal(again, fused)
