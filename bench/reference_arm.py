"""The unmodified reference library (``baseline/_ref/pcie_allreduce``) driven
through its own public API, for the benchmarks' reference arms.

Bootstrap as the reference's own scripts do it (bench_crossover.py:29-94):
CudaIPC buffers for the signal block and the two staging buffers, handle
exchange over a gloo group, ``init_custom_ar`` + ``register_pcie_buffers``;
calls go to ``pcie_allreduce.all_reduce``. CUDA graphs that captured it need
``post_capture()`` (its two-phase graph-buffer registration) on every rank.
"""

from __future__ import annotations

import contextlib
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def reference_available() -> bool:
    return os.path.isdir(os.path.join(REF_DIR, "pcie_allreduce"))


@contextlib.contextmanager
def stdout_to_stderr():
    """Keeps build logs (the reference JIT-compiles on import) off stdout."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


class ReferenceArm:
    """The unmodified reference (baseline/_ref/pcie_allreduce) through its own
    public API, bootstrapped like its bench_crossover.py."""

    name = "reference"

    def __init__(self, rank, world, gloo, max_bytes):
        if not reference_available():
            raise RuntimeError("reference not installed under baseline/_ref")
        sys.path.insert(0, REF_DIR)
        with stdout_to_stderr():
            import pcie_allreduce  # noqa: F401  (JIT build happens here)
        from pcie_allreduce.cuda_ipc import CudaIPC

        self.ar = pcie_allreduce
        self.rank, self.world, self.gloo = rank, world, gloo
        ipc = CudaIPC()
        cap = max_bytes * world  # push path needs bytes * world <= capacity
        meta_sz = pcie_allreduce.meta_size()
        meta = ipc.malloc(meta_sz + cap)
        ipc.memset(meta, 0, meta_sz + cap)
        self._refs = []

        def exchange(ptr):
            hs = [None] * world
            dist.all_gather_object(hs, ipc.ipc_get_handle(ptr), group=gloo)
            out = []
            for i, h in enumerate(hs):
                if i == rank:
                    out.append(ptr.value)
                else:
                    p = ipc.ipc_open_handle(h)
                    self._refs.append(p)
                    out.append(p.value)
            return out

        meta_ptrs = exchange(meta)
        buf0 = exchange(ipc.malloc(cap))
        buf1 = exchange(ipc.malloc(cap))
        self.rank_data = torch.empty(8 << 20, dtype=torch.uint8, device="cuda")
        self.fa = pcie_allreduce.init_custom_ar(meta_ptrs, self.rank_data, rank)
        pcie_allreduce.register_pcie_buffers(self.fa, buf0, buf1, cap)
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        self.n = 0

    def all_reduce(self, inp, out):
        self.ar.all_reduce(self.fa, inp, out, 0, 0)
        self.n += 1

    def post_capture(self):
        handle, off = self.ar.get_graph_buffer_ipc_meta(self.fa)
        meta = [None] * self.world
        dist.all_gather_object(meta, (handle, off), group=self.gloo)
        self.ar.register_graph_buffers(self.fa, [m[0] for m in meta], [m[1] for m in meta])
        dist.barrier(group=self.gloo)

    def launches(self):
        return self.n  # one kernel per call (cu:425-476)

    def variant(self, nbytes):
        return "reference"

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(group=self.gloo)
