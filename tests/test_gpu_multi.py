"""Multi-GPU tests (one process per GPU, NCCL + gloo groups): every variant,
dtype and a range of sizes against an fp32 oracle, CUDA-graph replays, the
zero-copy registered path, the reference-compatible op set, and a stress run
in the style of the reference's stress_test.py."""

import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0
if NGPU < 2:
    pytest.skip("needs at least two GPUs", allow_module_level=True)
WORLD = min(NGPU, 8)

VARIANTS = ["oneshot_push", "oneshot_pull", "twoshot", "twoshot_push", "lamport"]


def _oracle(x, world):
    """fp32 sum in rank order, as the kernels accumulate."""
    xs = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(xs, x)
    acc = xs[0].float()
    for t in xs[1:]:
        acc = acc + t.float()
    return acc


def _comm(rank, **kw):
    from b200ar import CustomAllreduce

    gloo = dist.new_group(backend="gloo")
    return CustomAllreduce(group=gloo, device=torch.device("cuda", rank), nccl_group=dist.group.WORLD, **kw)


def _variants_dtypes(rank, world):
    comm = _comm(rank, max_size=8 << 20)
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        per16 = 16 // torch.tensor([], dtype=dtype).element_size()
        for numel in (per16, 5 * per16, 7168, 7168 * 3, 1 << 20, (1 << 20) + 9 * per16):
            g = torch.Generator(device="cuda").manual_seed(1234 + rank + numel)
            x = (torch.rand(numel, generator=g, device="cuda") * 2 - 1).to(dtype)
            ref = _oracle(x, world).to(dtype)
            for variant in VARIANTS + ["auto"]:
                nbytes = numel * x.element_size()
                if variant == "oneshot_push" and nbytes * world > comm.slot_capacity:
                    continue
                if variant == "lamport" and nbytes > comm.lamport_capacity:
                    continue
                for ctas in (0, 1, 7):
                    out = comm.all_reduce(x, variant=variant, ctas=ctas)
                    torch.cuda.synchronize()
                    assert torch.equal(out, ref), (dtype, numel, variant, ctas,
                                                   (out.float() - ref.float()).abs().max().item())
    comm.check()
    comm.close()


def test_variants_dtypes_sizes():
    run_ranks(_variants_dtypes, WORLD, backend="nccl")


def _graph_replay(rank, world):
    # Slot variants inside a CUDA graph: the slot and epochs come from the device
    # generation counter, so replays alternate buffers without any registration.
    comm = _comm(rank, max_size=8 << 20)
    inp = torch.zeros(7168, device="cuda", dtype=torch.bfloat16)
    mid = torch.empty_like(inp)
    out = torch.empty_like(inp)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        comm.all_reduce(inp, mid)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for variant in ("oneshot_push", "twoshot", "twoshot_push", "oneshot_pull", "lamport"):
            comm.all_reduce(inp, mid, variant=variant)
            mid.mul_(1.0 / world)
            comm.all_reduce(mid, out, variant=variant)
    for i in range(200):
        inp.fill_(float(rank + 1) + (i % 7))
        g.replay()
    torch.cuda.synchronize()
    want = sum(float(r + 1) + (199 % 7) for r in range(world))
    assert torch.allclose(out.float(), torch.full_like(out.float(), want), rtol=2e-2), out[:4]
    comm.check()
    comm.close()


def test_graph_replay():
    run_ranks(_graph_replay, WORLD, backend="nccl")


def _registered_zero_copy(rank, world):
    # Zero-copy path: captured inputs are exchanged after capture (the
    # reference's two-phase protocol) and read in place by the peers.
    comm = _comm(rank, max_size=1 << 20)
    x = torch.zeros(1 << 16, device="cuda", dtype=torch.bfloat16)
    y = torch.empty_like(x)
    g = torch.cuda.CUDAGraph()
    with comm.capture():
        with torch.cuda.graph(g):
            comm.all_reduce(x, y, variant="registered")
    base = torch.arange(x.numel(), device="cuda").float().remainder(13)
    for i in range(50):
        x.copy_((base + rank + i).to(torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        ref = _oracle(x, world).to(torch.bfloat16)
        assert torch.equal(y, ref), i
    comm.check()
    comm.close()


def test_registered_zero_copy_graph():
    run_ranks(_registered_zero_copy, WORLD, backend="nccl")


def _compat_api(rank, world):
    # The reference's own bootstrap (test_pcie_ar.py / stress_test.py) against
    # b200ar.compat and b200ar.ipc.CudaIPC.
    import b200ar.compat as pcie_allreduce
    from b200ar.ipc import CudaIPC

    gloo = dist.new_group(backend="gloo")
    ipc = CudaIPC()
    max_size = 512 * 1024
    meta_sz = pcie_allreduce.meta_size()
    meta = ipc.malloc(meta_sz + max_size)
    ipc.memset(meta, 0, meta_sz + max_size)

    def exchange(ptr):
        hs = [None] * world
        dist.all_gather_object(hs, ipc.ipc_get_handle(ptr), group=gloo)
        return [ptr.value if i == rank else ipc.ipc_open_handle(h).value for i, h in enumerate(hs)]

    meta_ptrs = exchange(meta)
    buf0, buf1 = exchange(ipc.malloc(max_size)), exchange(ipc.malloc(max_size))
    rank_data = torch.empty(max_size, dtype=torch.uint8, device="cuda")
    fa = pcie_allreduce.init_custom_ar(meta_ptrs, rank_data, rank)
    pcie_allreduce.register_pcie_buffers(fa, buf0, buf1, max_size)
    expected = world * (world + 1) / 2.0
    for dtype, n in ((torch.bfloat16, 7168), (torch.float16, 7168), (torch.float32, 512), (torch.bfloat16, 16)):
        inp = torch.full((1, n), float(rank + 1), dtype=dtype, device="cuda")
        out = torch.zeros_like(inp)
        for _ in range(100):
            pcie_allreduce.all_reduce(fa, inp, out, 0, 0)
        torch.cuda.synchronize()
        assert (out.float() - expected).abs().max().item() < 0.5
    # Graph capture through the compat API (stress_test.py t10 flow).
    g_inp = torch.full((1, 7168), float(rank + 1), dtype=torch.bfloat16, device="cuda")
    g_out = torch.zeros_like(g_inp)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(10):
            pcie_allreduce.all_reduce(fa, g_inp, g_out, 0, 0)
    handle, off = pcie_allreduce.get_graph_buffer_ipc_meta(fa)
    allm = [None] * world
    dist.all_gather_object(allm, (handle, off), group=gloo)
    pcie_allreduce.register_graph_buffers(fa, [m[0] for m in allm], [m[1] for m in allm])
    for _ in range(100):
        g_inp.fill_(float(rank + 1))
        g.replay()
    torch.cuda.synchronize()
    assert (g_out.float() - expected).abs().max().item() < 0.5
    # A message larger than the registered capacity is rejected, not overflowed.
    big = torch.ones(max_size, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        pcie_allreduce.all_reduce(fa, big, torch.empty_like(big), 0, 0)
    torch.cuda.synchronize()
    dist.barrier(group=gloo)
    pcie_allreduce.dispose(fa)


def test_compat_api():
    run_ranks(_compat_api, WORLD, backend="nccl")


def _stress(rank, world):
    # Alternating sizes and variants back to back with values that change every
    # call (stress_test.py t4/t5/t8), checked every 97 calls and at the end.
    comm = _comm(rank, max_size=4 << 20)
    gen = torch.Generator().manual_seed(99)
    sizes = [16, 7168, 7168 * 4, 1 << 16, (1 << 20) + 8]
    last = None
    for i in range(3000):
        n = sizes[int(torch.randint(len(sizes), (1,), generator=gen))]
        v = float(rank + 1) + (i % 11) * 0.125
        x = torch.full((n,), v, dtype=torch.float32, device="cuda")
        out = comm.all_reduce(x, variant="lamport" if (i % 3 == 0 and n * 4 <= comm.lamport_capacity) else "auto")
        last = (out, sum(float(r + 1) + (i % 11) * 0.125 for r in range(world)))
        if i % 97 == 0:
            torch.cuda.synchronize()
            assert torch.all(out == last[1]), i
    torch.cuda.synchronize()
    assert torch.all(last[0] == last[1])
    comm.check()
    comm.close()


def test_stress_mixed_sizes():
    run_ranks(_stress, WORLD, backend="nccl")


def _fused_rmsnorm(rank, world):
    # Benchmark shapes: partial [T, 8192] ~ N(0,1), residual ~ N(0,1),
    # gamma = 1 + 0.01 N(0,1), eps 1e-5, T in {1, 8, 32, 128, 512}.
    from b200ar.ops.fused import ref_ar_residual_rmsnorm

    comm = _comm(rank, max_size=32 << 20)
    H = 8192
    g0 = torch.Generator(device="cuda").manual_seed(7)
    gamma = (1 + 0.01 * torch.randn(H, generator=g0, device="cuda")).to(torch.bfloat16)
    for T in (1, 8, 32, 128, 512):
        g = torch.Generator(device="cuda").manual_seed(1234 + rank + 17 * T)
        x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
        res = torch.randn(T, H, generator=torch.Generator(device="cuda").manual_seed(55 + T),
                          device="cuda").to(torch.bfloat16)
        xs = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(xs, x)
        y_ref, z_ref = ref_ar_residual_rmsnorm(xs, res, gamma, 1e-5)
        for variant in ("oneshot_push", "twoshot", "lamport", "auto"):
            y, z = comm.all_reduce_residual_rmsnorm(x, res, gamma, 1e-5, variant=variant)
            torch.cuda.synchronize()
            assert torch.equal(z, z_ref), (T, variant)
            torch.testing.assert_close(y.float(), y_ref.float(), atol=2e-2, rtol=1e-2)
        # In-place residual update.
        r2 = res.clone()
        y, z = comm.all_reduce_residual_rmsnorm(x, r2, gamma, 1e-5, residual_out=r2)
        torch.cuda.synchronize()
        assert z.data_ptr() == r2.data_ptr() and torch.equal(r2, z_ref)
    comm.check()
    comm.close()


def test_fused_allreduce_residual_rmsnorm():
    run_ranks(_fused_rmsnorm, WORLD, backend="nccl")


def _nvls(rank, world):
    # NVLS is opt-in; the buffer is always released (a process that exits with
    # memory bound to a multicast object can fault the peers).
    comm = _comm(rank, max_size=64 << 20, enable_nvls=True)
    try:
        if comm.nvls is None:
            return
        for dtype in (torch.bfloat16, torch.float32):
            for numel in (8 * 1024, 1 << 20, 16 << 20):
                if numel * torch.tensor([], dtype=dtype).element_size() > (64 << 20):
                    continue
                g = torch.Generator(device="cuda").manual_seed(rank + numel)
                x = (torch.rand(numel, generator=g, device="cuda") * 2 - 1).to(dtype)
                ref = _oracle(x, world)
                for _ in range(3):
                    out = comm.all_reduce(x, variant="nvls")
                    torch.cuda.synchronize()
                    torch.testing.assert_close(out.float(), ref, atol=2e-2 * world, rtol=1e-2)
                # Every rank receives the same multicast value.
                outs = [torch.empty_like(out) for _ in range(world)]
                dist.all_gather(outs, out)
                assert all(torch.equal(o, outs[0]) for o in outs)
        comm.check()
    finally:
        comm.close()


def test_nvls_multimem():
    run_ranks(_nvls, WORLD, backend="nccl")


def _gemm_allreduce(rank, world):
    # (down projection): x [M, 3584] ~ N(0,1), W [8192, 3584] ~ N(0, 0.02).
    from b200ar.ops.gemm import check_errors, error_word

    comm = _comm(rank, max_size=160 << 20)
    K, N = 3584, 8192
    for M in (16, 128, 1024):
        g = torch.Generator(device="cuda").manual_seed(1234 + rank + M)
        x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
        w = (0.02 * torch.randn(N, K, generator=g, device="cuda")).to(torch.bfloat16)
        part = (x.float() @ w.float().t())
        ref = part.clone()
        dist.all_reduce(ref)
        for fused in (True, False):
            for _ in range(2):
                out = comm.linear_all_reduce(x, w, fused=fused) if not fused else torch.empty_like(ref).to(
                    torch.bfloat16)
                if fused:
                    comm._comm.gemm_allreduce(x, w, out, error_word(x.device))
                torch.cuda.synchronize()
                check_errors()
                err = (out.float() - ref).abs().max().item()
                assert err <= 2e-2 * ref.abs().max().item() + 2e-2, (M, fused, err)
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        assert all(torch.equal(o, outs[0]) for o in outs), "ranks disagree"
    comm.check()
    comm.close()


def test_gemm_allreduce_fused():
    run_ranks(_gemm_allreduce, WORLD, backend="nccl")


def _ag_gemm(rank, world):
    from b200ar.ops.gemm import check_errors

    comm = _comm(rank, max_size=64 << 20)
    K, N = 8192, 3584
    for rows in (16, 128, 512):
        g = torch.Generator(device="cuda").manual_seed(99 + rank + rows)
        x = torch.randn(rows, K, generator=g, device="cuda").to(torch.bfloat16)
        w = (0.02 * torch.randn(N, K, generator=torch.Generator(device="cuda").manual_seed(5 + rank),
                                device="cuda")).to(torch.bfloat16)
        full = torch.empty(rows * world, K, dtype=torch.bfloat16, device="cuda")
        dist.all_gather_into_tensor(full, x)
        ref = full.float() @ w.float().t()
        for _ in range(3):
            y = comm.all_gather_linear(x, w)
            torch.cuda.synchronize()
            check_errors()
            err = (y.float() - ref).abs().max().item()
            assert err <= 1e-2 * ref.abs().max().item() + 1e-2, (rows, err)
        # Interleave with all-reduces (shared generation / slots).
        comm.all_reduce(x)
    comm.check()
    comm.close()


def test_allgather_gemm_fused():
    run_ranks(_ag_gemm, WORLD, backend="nccl")


def _nccl_crossover_paths(rank, world):
    # Above the NCCL crossover: in-place calls run NCCL's all-reduce,
    # out-of-place calls NCCL's reduce-scatter into the output's shard plus an
    # in-place all-gather (no extra copy); both must give the sum.
    comm = _comm(rank, max_size=8 << 20)
    comm.set_selector([(1 << 62, "nccl", 0)])
    x = (torch.rand(1 << 20, device="cuda") * 2 - 1).to(torch.bfloat16)
    ref = _oracle(x, world)
    n0 = comm.launches
    out = comm.all_reduce(x)
    torch.cuda.synchronize()
    assert comm.launches == n0  # NCCL, none of our kernels
    torch.testing.assert_close(out.float(), ref, atol=2e-2 * world, rtol=1e-2)
    y = x.clone()
    comm.all_reduce(y, out=y)
    torch.cuda.synchronize()
    assert comm.launches == n0  # NCCL in place
    torch.testing.assert_close(y.float(), ref, atol=2e-2 * world, rtol=1e-2)
    comm.close()


def test_nccl_crossover_paths():
    run_ranks(_nccl_crossover_paths, WORLD, backend="nccl")
