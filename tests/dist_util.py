"""Helpers to run a test body on several ranks (one process each)."""

import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, backend, fn, args, errq):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    try:
        if backend == "nccl":
            torch.cuda.set_device(rank)
        dist.init_process_group(backend, rank=rank, world_size=world)
        fn(rank, world, *args)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:  # noqa: BLE001 - reported to the parent
        errq.put((rank, traceback.format_exc()))
        raise


def run_ranks(fn, world, *args, backend="gloo", timeout=600):
    """Runs ``fn(rank, world, *args)`` on ``world`` spawned processes after
    ``init_process_group(backend)``; raises with the first rank's traceback."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, backend, fn, args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    if errors:
        rank, tb = sorted(errors)[0]
        raise AssertionError(f"rank {rank} failed:\n{tb}")
    if alive:
        raise AssertionError(f"{len(alive)} rank(s) did not finish within {timeout}s")
    bad = [p.exitcode for p in procs if p.exitcode != 0]
    if bad:
        raise AssertionError(f"rank exit codes {bad}")
