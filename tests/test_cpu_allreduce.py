"""CPU (gloo bootstrap + shared-memory data plane) tests of the all-reduce
protocol: the same layout, epochs, slots and algorithms as the GPU kernels."""

import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks

VARIANTS = ["oneshot_push", "oneshot_pull", "twoshot", "twoshot_push", "lamport"]


def _bf16_1024x1024_fp32_oracle(rank, world):
    # Benchmark configuration: bf16 [1024, 1024] ~ N(0, 1) seeded 1234 + rank, fp32 oracle, atol 2e-2.
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(group=None, device="cpu", max_size=4 << 20)
    inputs = []
    for r in range(world):
        g = torch.Generator().manual_seed(1234 + r)
        inputs.append(torch.randn(1024, 1024, generator=g).to(torch.bfloat16))
    ref = sum(x.float() for x in inputs)
    for variant in VARIANTS:
        out = comm.all_reduce(inputs[rank], variant=variant)
        err = (out.float() - ref).abs()
        # fp32 accumulation, one bf16 rounding of the result: within atol 2e-2
        # plus half an ulp of bf16 (2^-9 relative).
        assert bool((err <= 2e-2 + ref.abs() * 2.0**-8).all()), (variant, float(err.max()))
        assert torch.equal(out, ref.to(torch.bfloat16)), variant
    comm.close()


def test_bf16_1024x1024_fp32_oracle_gloo_ws2():
    run_ranks(_bf16_1024x1024_fp32_oracle, 2)


def _dtypes_sizes(rank, world):
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 20)
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        per16 = 16 // torch.tensor([], dtype=dtype).element_size()
        for numel in (per16, 3 * per16, 7168, 14336, 65536 + per16):
            for variant in VARIANTS:
                for ctas in (1, 3, 8):
                    g = torch.Generator().manual_seed(numel * 7 + rank)
                    x = (torch.rand(numel, generator=g) * 2 - 1).to(dtype)
                    xs = [None] * world
                    dist.all_gather_object(xs, x)
                    ref = sum(t.float() for t in xs)
                    out = comm.all_reduce(x, variant=variant, ctas=ctas)
                    torch.testing.assert_close(out, ref.to(dtype), rtol=0, atol=0)
    comm.close()


@pytest.mark.parametrize("world", [2, 3, 4, 6])
def test_dtypes_sizes_variants(world):
    run_ranks(_dtypes_sizes, world)


def _many_calls(rank, world):
    # Back-to-back calls alternate the double-buffer slot; values change every
    # call, so a slot reused too early would corrupt results (reference t4/t5).
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 20)
    for i in range(300):
        numel = 16 if i % 2 == 0 else 7168
        variant = VARIANTS[i % len(VARIANTS)]
        x = torch.full((numel,), float(rank + 1) + i * 0.25, dtype=torch.float32)
        out = comm.all_reduce(x, variant=variant, ctas=1 + i % 4)
        want = sum(float(r + 1) + i * 0.25 for r in range(world))
        assert torch.all(out == want), (i, variant, out[:4])
    assert comm._shm.generation == 300
    comm.close()


def test_many_calls_slot_alternation():
    run_ranks(_many_calls, 2)


def _in_place(rank, world):
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 20)
    for variant in VARIANTS:
        x = torch.arange(4096, dtype=torch.float32) + rank
        comm.all_reduce(x, out=x, variant=variant)
        want = torch.arange(4096, dtype=torch.float32) * world + sum(range(world))
        assert torch.equal(x, want), variant
    comm.close()


def test_in_place():
    run_ranks(_in_place, 2)


def _timeout_and_reset(rank, world):
    from b200ar import CommTimeoutError, CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 20, timeout_ms=200)
    x = torch.ones(1024)
    comm.all_reduce(x)
    # Rank 1 skips the barrier of the next call: rank 0 must time out, not hang.
    if rank == 1:
        comm._shm.inject_skip(1)
    raised = False
    try:
        comm.all_reduce(x, variant="oneshot_pull")
    except CommTimeoutError as e:
        raised = True
        assert "timed out" in str(e)
    flags = [None] * world
    dist.all_gather_object(flags, raised)
    assert flags[0] is True and flags[1] is False, flags
    # A communicator in error state refuses work until it is reset collectively.
    if rank == 0:
        with pytest.raises(CommTimeoutError):
            comm.all_reduce(x)
    comm.reset()
    out = comm.all_reduce(torch.full((2048,), float(rank)), variant="twoshot")
    assert torch.all(out == sum(range(world)))
    # A Lamport call whose peer never writes also times out; after reset the
    # buffers hold markers again and Lamport calls give exact sums.
    if rank == 1:
        comm._shm.inject_skip(1)
    try:
        comm.all_reduce(x, variant="lamport")
    except CommTimeoutError:
        pass
    dist.barrier()
    comm.reset()
    for i in range(6):
        out = comm.all_reduce(torch.full((4096,), float(rank + i)), variant="lamport")
        assert torch.all(out == sum(r + i for r in range(world))), i
    comm.close()


def test_timeout_detection_and_reset():
    run_ranks(_timeout_and_reset, 2)


def _world1(rank, world):
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device="cpu")
    x = torch.randn(1000)
    assert torch.equal(comm.all_reduce(x), x)
    comm.close()


def test_world_size_one():
    run_ranks(_world1, 1)


def _fused_cpu(rank, world):
    from b200ar import CustomAllreduce
    from b200ar.ops.fused import ref_ar_residual_rmsnorm

    comm = CustomAllreduce(device="cpu", max_size=1 << 20)
    H = 1024
    x = torch.randn(4, H, generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16)
    res = torch.randn(4, H, generator=torch.Generator().manual_seed(99)).to(torch.bfloat16)
    gamma = torch.ones(H, dtype=torch.bfloat16)
    xs = [None] * world
    dist.all_gather_object(xs, x)
    y_ref, z_ref = ref_ar_residual_rmsnorm(xs, res, gamma)
    y, z = comm.all_reduce_residual_rmsnorm(x, res, gamma)
    assert torch.equal(z, z_ref)
    torch.testing.assert_close(y.float(), y_ref.float(), atol=2e-2, rtol=1e-2)
    comm.close()


def test_fused_residual_rmsnorm_cpu():
    run_ranks(_fused_cpu, 2)


def _dead_peer(rank, world):
    # Rank 1 leaves after set-up without ever calling the collective: rank 0's
    # barrier must end in a CommTimeoutError (bounded wait), not a hang.
    import time

    from b200ar import CommTimeoutError, CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 20, timeout_ms=300)
    if rank == 1:
        return
    t0 = time.time()
    with pytest.raises(CommTimeoutError):
        comm.all_reduce(torch.ones(4096), variant="twoshot")
    assert time.time() - t0 < 10


def test_dead_peer_times_out():
    import torch.multiprocessing as mp  # noqa: F401

    from dist_util import run_ranks as _run

    # The surviving rank must not wait on a barrier of the process group at exit.
    _run(_dead_peer_entry, 2)


def _dead_peer_entry(rank, world):
    import torch.distributed as dist

    _dead_peer(rank, world)
    # Skip the final dist.barrier() of the harness for the departed rank: both
    # ranks meet here once rank 0 observed the timeout.
    dist.barrier()


def _ragged(rank, world):
    # Sizes that are not a multiple of 16 bytes, misaligned views and strided
    # tensors go through a padded staging copy; results stay exact.
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 20)
    for dtype in (torch.float32, torch.bfloat16):
        for numel in (1, 7, 13, 1025):
            g = torch.Generator().manual_seed(numel + 31 * rank)
            base = (torch.rand(3 * numel + 3, generator=g) * 2 - 1).to(dtype)
            for name, x in (("plain", base[:numel].clone()), ("misaligned", base[1:1 + numel]),
                            ("strided", base[::3][:numel])):
                xs = [None] * world
                dist.all_gather_object(xs, x.clone())
                ref = sum(t.float() for t in xs).to(dtype)
                out = comm.all_reduce(x)
                assert torch.equal(out, ref), (dtype, numel, name)
                y = torch.empty(3 * numel, dtype=dtype)[::3]  # strided output
                comm.all_reduce(x, out=y)
                assert torch.equal(y, ref), (dtype, numel, name, "strided out")
    with pytest.raises(TypeError):
        comm.all_reduce(torch.ones(5, dtype=torch.int32))
    comm.close()


def test_ragged_misaligned_strided():
    run_ranks(_ragged, 2)


def _engine_interface(rank, world):
    from b200ar import CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 16)
    x = torch.full((1024,), float(rank + 1))
    assert not comm.disabled
    assert comm.should_custom_ar(x)
    out = comm.custom_all_reduce(x)
    assert out is not None and out.data_ptr() != x.data_ptr()
    assert torch.all(out == sum(r + 1 for r in range(world)))
    big = torch.zeros((1 << 16) // 4 + 4)  # above max_size: the caller's NCCL path
    assert not comm.should_custom_ar(big) and comm.custom_all_reduce(big) is None
    assert not comm.should_custom_ar(torch.zeros(5, dtype=torch.int32))
    assert not comm.should_custom_ar(torch.zeros(7, dtype=torch.bfloat16))  # 14 bytes
    comm.close()
    assert comm.disabled and not comm.should_custom_ar(x)


def test_serving_engine_interface():
    run_ranks(_engine_interface, 2)
