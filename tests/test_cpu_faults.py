"""Host-side fault injection beyond barrier timeouts (no GPU involved):

* a signal block overwritten with an epoch the protocol never writes is
  detected at the barrier, the call raises, and ``reset()`` recovers;
* a corrupted or mismatched segment exchange is rejected when the peer
  segment is mapped, before any data moves;
* the checked debug build (device-side range and epoch checks,
  ``-DB200AR_CHECKS``) compiles for sm_100a.
"""

import os
import shutil
import subprocess
import uuid

import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STATUS_BAD_EPOCH = 3


def _stale_epoch(rank, world):
    from b200ar import CommTimeoutError, CustomAllreduce

    comm = CustomAllreduce(device="cpu", max_size=1 << 20, timeout_ms=2000)
    x = torch.ones(1024)
    assert torch.all(comm.all_reduce(x, variant="oneshot_pull", ctas=1) == world)
    dist.barrier()
    # Rank 0's flag from rank 1 (CTA 0) is overwritten with an epoch far ahead
    # of anything the protocol writes; rank 1 sits out the next barrier so the
    # value stays in place. Without the check rank 0 would take the flag as an
    # arrival and read a slot rank 1 never filled.
    if rank == 0:
        comm._shm.inject_flag(0, 1, 1000)
    else:
        comm._shm.inject_skip(1)
    dist.barrier()
    raised = None
    try:
        comm.all_reduce(x, variant="oneshot_pull", ctas=1)
    except CommTimeoutError as e:
        raised = str(e)
    if rank == 0:
        assert raised is not None and "never writes" in raised, raised
        assert comm.status()["code"] == STATUS_BAD_EPOCH
        with pytest.raises(CommTimeoutError):  # error state until reset
            comm.all_reduce(x)
    else:
        assert raised is None
    comm.reset()
    for variant in ("oneshot_pull", "oneshot_push", "twoshot"):
        out = comm.all_reduce(torch.full((4096,), float(rank + 1)), variant=variant, ctas=2)
        assert torch.all(out == sum(r + 1 for r in range(world))), variant
    comm.close()


def test_stale_epoch_detected_and_reset():
    run_ranks(_stale_epoch, 2)


def test_corrupted_exchange_rejected():
    from b200ar import _C

    tag = uuid.uuid4().hex[:10]
    r0 = _C.ShmComm(f"/b200ar-t{tag}a", 0, 2, 4096, 1024)
    r1 = _C.ShmComm(f"/b200ar-t{tag}b", 1, 2, 4096, 1024)
    other = _C.ShmComm(f"/b200ar-t{tag}c", 1, 2, 8192, 1024)  # different capacity
    wrong_rank = _C.ShmComm(f"/b200ar-t{tag}d", 0, 2, 4096, 1024)  # same size, owner rank 0
    try:
        with pytest.raises(RuntimeError, match="shm_open"):
            r0.connect([r0.segment_name, f"/b200ar-t{tag}-missing"])
        with pytest.raises(RuntimeError, match="bytes, expected"):
            r0.connect([r0.segment_name, other.segment_name])
        with pytest.raises(RuntimeError, match="corrupted or mismatched"):
            r0.connect([r0.segment_name, wrong_rank.segment_name])
        with pytest.raises(ValueError, match="own segment"):
            r0.connect([r1.segment_name, r1.segment_name])
        # The correct exchange still connects, in both directions.
        r0.connect([r0.segment_name, r1.segment_name])
        r1.connect([r0.segment_name, r1.segment_name])
        # reset() keeps the header: a peer connecting afterwards still validates.
        r1.reset()
        r0.connect([r0.segment_name, r1.segment_name])
    finally:
        del r0, r1, other, wrong_rank


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc")
@pytest.mark.parametrize("src", ["csrc/comm/ar_kernels.cu", "csrc/comm/communicator.cu"])
def test_checked_build_compiles(src, tmp_path):
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-DB200AR_CHECKS", "-I", os.path.join(ROOT, "csrc"), "-c", os.path.join(ROOT, src), "-o",
           str(tmp_path / "k.o")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-3000:]
