"""Single-GPU tests: world size 1, IPC helpers, and the bounded barrier (a
flag that nothing sets must end in a reported timeout, never a hang)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)


def _lib():
    from b200ar import _C

    return _C


def test_native_library_is_loaded():
    import b200ar

    assert b200ar._C.__file__.endswith(".so")
    assert b200ar._C.meta_size() == b200ar._C.SIGNAL_BYTES


def test_ipc_helpers_roundtrip():
    from b200ar.ipc import CudaIPC, cudaIpcMemHandle_t

    ipc = CudaIPC()
    p = ipc.malloc(1 << 20)
    ipc.memset(p, 7, 1 << 20)
    h = ipc.ipc_get_handle(p)
    assert isinstance(h, cudaIpcMemHandle_t) and len(h.to_bytes()) == 64
    base, size = _lib().allocation_range(p.value + 4096)
    assert base == p.value and size >= 1 << 20
    ipc.free(p)


def _local_comm(world, cap=1 << 20, timeout_ms=20):
    """Communicator whose 'peer' workspaces are further local allocations that
    no kernel ever signals: every barrier must time out."""
    C = _lib()
    ws = [C.ipc_malloc(C.workspace_bytes(cap)) for _ in range(world)]
    rank_data = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")
    comm = C.Comm(ws, rank_data, 0)
    sig = C.SIGNAL_BYTES
    comm.register_slots([p + sig for p in ws], [p + sig + cap for p in ws], cap)
    lam = [C.ipc_malloc(C.lamport_bytes(1 << 16, world)) for _ in range(world)]
    comm.register_lamport(lam, 1 << 16)
    ws = ws + lam
    comm.set_timeout_ns(timeout_ms * 1_000_000)
    return comm, ws, rank_data


@pytest.mark.parametrize("variant", ["oneshot_push", "oneshot_pull", "twoshot", "lamport"])
def test_barrier_timeout_reports_status(variant):
    from b200ar import CommTimeoutError
    from b200ar.parallel.selector import VARIANTS

    comm, ws, _rd = _local_comm(2)
    x = torch.randn(4096, device="cuda", dtype=torch.bfloat16)
    y = torch.empty_like(x)
    comm.all_reduce(x, y, VARIANTS[variant], 2)
    torch.cuda.synchronize()  # returns: the wait is bounded
    st = comm.status()
    assert st["code"] == 1 and st["peer"] == 1 and st["rank"] == 0, st
    with pytest.raises(CommTimeoutError):
        comm.check()
    with pytest.raises(CommTimeoutError):
        comm.all_reduce(x, y, VARIANTS[variant], 2)
    comm.reset()
    assert comm.status()["code"] == 0
    del comm
    for p in ws:
        _lib().ipc_free(p)


def test_world_one_copy_and_launch_count():
    import torch.distributed as dist

    from dist_util import free_port

    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device=torch.device("cuda", 0), max_size=1 << 20)
    x = torch.randn(7168, device="cuda", dtype=torch.bfloat16)
    n0 = comm.launches
    y = comm.all_reduce(x)
    torch.cuda.synchronize()
    assert torch.equal(x, y)
    assert comm.launches == n0 + 1
    comm.close()
    dist.destroy_process_group()


def test_fused_rmsnorm_world_one():
    import torch.distributed as dist

    from dist_util import free_port

    from b200ar import CustomAllreduce
    from b200ar.ops.fused import ref_ar_residual_rmsnorm

    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    comm = CustomAllreduce(device=torch.device("cuda", 0), max_size=8 << 20)
    for H in (4096, 8192, 16384):
        x = torch.randn(33, H, device="cuda").to(torch.bfloat16)
        res = torch.randn(33, H, device="cuda").to(torch.bfloat16)
        gamma = (1 + 0.01 * torch.randn(H, device="cuda")).to(torch.bfloat16)
        y, z = comm.all_reduce_residual_rmsnorm(x, res, gamma, 1e-5)
        y_ref, z_ref = ref_ar_residual_rmsnorm([x], res, gamma, 1e-5)
        assert torch.equal(z, z_ref)
        torch.testing.assert_close(y.float(), y_ref.float(), atol=2e-2, rtol=1e-2)
    comm.close()
    dist.destroy_process_group()


def test_torch_ops_match_eager_paths():
    """torch.ops.b200ar (direct and traced by torch.compile) gives bitwise the
    results of the pybind entry points: same kernels, same streams."""
    import torch.distributed as dist

    from dist_util import free_port

    from b200ar import CustomAllreduce
    from b200ar.ops.layers import rmsnorm, silu_mul

    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    comm = CustomAllreduce(device=torch.device("cuda", 0), max_size=8 << 20)
    assert comm.handle != 0
    H = 4096
    x = torch.randn(33, H, device="cuda").to(torch.bfloat16)
    res = torch.randn(33, H, device="cuda").to(torch.bfloat16)
    gamma = (1 + 0.01 * torch.randn(H, device="cuda")).to(torch.bfloat16)

    def layer(x, res, g):
        s = comm.all_reduce(x)
        y, z = comm.all_reduce_residual_rmsnorm(s, res, g, 1e-5)
        return silu_mul(torch.cat([rmsnorm(y, g, 1e-5), z], dim=1))

    ref = layer(x, res, gamma)
    s = torch.empty_like(x)
    torch.ops.b200ar.all_reduce(comm.handle, x, s)
    y = torch.empty_like(x)
    z = torch.empty_like(x)
    torch.ops.b200ar.all_reduce_residual_rmsnorm(comm.handle, s, res, gamma, 1e-5, y, z)
    y_ref, z_ref = comm.all_reduce_residual_rmsnorm(x, res, gamma, 1e-5)
    torch.cuda.synchronize()
    assert torch.equal(s, x) and torch.equal(y, y_ref) and torch.equal(z, z_ref)
    torch._dynamo.reset()
    out = torch.compile(layer, fullgraph=True, backend="aot_eager")(x, res, gamma)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    comm.close()
    dist.destroy_process_group()
