"""GPU test of the allocation-free residual-add + RMSNorm entry point.

Callers such as inference-engine plugins may not allocate device memory while
they run, so b200ar exports ``b200ar_residual_rmsnorm_noalloc``, a C function
that takes inputs and outputs only and keeps its scratch in an array built
into the library. This test calls that exported C symbol through ctypes and
checks it against the regular entry point (``CustomAllreduce`` with one rank,
whose scratch lives in a workspace it allocates) and against the plain fp32
PyTorch reference, on two calls in a row, and checks that a call allocates no
device memory.
The file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)


def _lib():
    import b200ar

    lib = ctypes.CDLL(b200ar._C.__file__)
    f = lib.b200ar_residual_rmsnorm_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p]
    lib.b200ar_noalloc_last_error.restype = ctypes.c_char_p
    return lib


def _call(lib, x, res, gamma, y, z, eps):
    rows, hidden = x.shape
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.b200ar_residual_rmsnorm_noalloc(x.data_ptr(), res.data_ptr(), gamma.data_ptr(), y.data_ptr(),
                                             z.data_ptr(), rows, hidden, ctypes.c_float(eps), stream)
    assert rc == 0, lib.b200ar_noalloc_last_error().decode()


def test_noalloc_matches_regular_entry_point():
    import torch.distributed as dist

    from dist_util import free_port

    from b200ar import CustomAllreduce
    from b200ar.ops.fused import ref_ar_residual_rmsnorm

    owns_pg = not dist.is_initialized()
    if owns_pg:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    comm = CustomAllreduce(device=torch.device("cuda", 0), max_size=8 << 20)
    lib = _lib()
    eps = 1e-5
    # (128, 8192) is exactly the 2 MiB limit.
    for rows, hidden in ((1, 8192), (32, 8192), (64, 4096), (128, 8192)):
        gamma = (1 + 0.01 * torch.randn(hidden, device="cuda")).to(torch.bfloat16)
        for call in range(2):  # two calls in a row share (and reuse) the scratch array
            x = torch.randn(rows, hidden, device="cuda").to(torch.bfloat16)
            res = torch.randn(rows, hidden, device="cuda").to(torch.bfloat16)
            y_ref, z_ref = comm.all_reduce_residual_rmsnorm(x, res, gamma, eps)
            y_f32, z_f32 = ref_ar_residual_rmsnorm([x], res, gamma, eps)
            y = torch.empty_like(x)
            z = torch.empty_like(x)
            _call(lib, x, res, gamma, y, z, eps)
            torch.cuda.synchronize()
            assert torch.equal(z, z_ref) and torch.equal(z, z_f32), (rows, hidden, call)
            torch.testing.assert_close(y.float(), y_ref.float(), atol=2e-2, rtol=1e-2)
            torch.testing.assert_close(y.float(), y_f32.float(), atol=2e-2, rtol=1e-2)
    comm.close()
    if owns_pg:
        dist.destroy_process_group()


def test_noalloc_rejects_oversized_request():
    lib = _lib()
    rows, hidden = 256, 8192  # 4 MiB > 2 MiB limit
    x = torch.zeros(rows, hidden, device="cuda", dtype=torch.bfloat16)
    gamma = torch.ones(hidden, device="cuda", dtype=torch.bfloat16)
    rc = lib.b200ar_residual_rmsnorm_noalloc(x.data_ptr(), x.data_ptr(), gamma.data_ptr(), x.data_ptr(),
                                             x.data_ptr(), rows, hidden, ctypes.c_float(1e-5),
                                             torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"exceeds" in lib.b200ar_noalloc_last_error()


def test_noalloc_call_allocates_nothing():
    lib = _lib()
    rows, hidden = 128, 8192
    x = torch.randn(rows, hidden, device="cuda").to(torch.bfloat16)
    res = torch.randn(rows, hidden, device="cuda").to(torch.bfloat16)
    gamma = torch.ones(hidden, device="cuda", dtype=torch.bfloat16)
    y = torch.empty_like(x)
    z = torch.empty_like(x)
    _call(lib, x, res, gamma, y, z, 1e-5)  # the first call on a device does its one-time set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        _call(lib, x, res, gamma, y, z, 1e-5)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == alloc0
    assert free1 == free0


def test_noalloc_rejects_rows_that_would_overflow():
    lib = _lib()
    x = torch.zeros(8, 8192, device="cuda", dtype=torch.bfloat16)
    gamma = torch.ones(8192, device="cuda", dtype=torch.bfloat16)
    rows = (1 << 62) // 8192 + 1  # rows * hidden * 2 wraps around in 64 bits
    rc = lib.b200ar_residual_rmsnorm_noalloc(x.data_ptr(), x.data_ptr(), gamma.data_ptr(), x.data_ptr(),
                                             x.data_ptr(), rows, 8192, ctypes.c_float(1e-5),
                                             torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and b"exceeds" in lib.b200ar_noalloc_last_error()
