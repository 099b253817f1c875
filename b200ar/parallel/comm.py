"""``CustomAllreduce``: the idiomatic b200ar communicator.

One object per rank (one process per GPU). Construction is collective over a
``torch.distributed`` group: it allocates this rank's workspace (signal block +
two message slots) with ``cudaMalloc``, exchanges CUDA IPC handles with
``all_gather_object``, maps the peers' workspaces and builds the native
communicator. This is the bootstrap that every reference script duplicates by
hand (test_pcie_ar.py:25-65, stress_test.py:26-77, bench_crossover.py:29-94).

For CPU tensors (``device="cpu"``) the same API runs on the shared-memory
emulation of the protocol (``_C.ShmComm``), bootstrapped over a gloo group.
"""

from __future__ import annotations

import contextlib
import uuid
from typing import List, Optional

import torch
import torch.distributed as dist

from .._native import _C
from ..config import Config, default_config
from ..log import logger
from . import selector as sel

CommTimeoutError = getattr(_C, "CommTimeout", RuntimeError)


class CustomAllreduce:
    """Sum all-reduce over NVLink/NVSwitch with custom sm_100a kernels.

    Args:
        group: process group used for bootstrap (handle exchange). Any backend
            that supports object collectives (gloo recommended).
        device: this rank's device (``torch.device``/index/``"cpu"``).
        nccl_group: optional NCCL group for the large-message fallback. When
            absent and ``group`` is an NCCL group, ``group`` is used.
        config: ``Config``; keyword overrides (``max_size=...``) are accepted too.
    """

    def __init__(self, group=None, device=None, nccl_group=None, config: Optional[Config] = None, **overrides):
        self.cfg = (config or default_config()).replace(**overrides) if overrides else (config or default_config())
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if nccl_group is None and group is not None and dist.get_backend(group) == "nccl":
            nccl_group = group
        if nccl_group is None and group is None and dist.is_initialized() and dist.get_backend() == "nccl":
            nccl_group = dist.group.WORLD
        self.nccl_group = nccl_group
        self.closed = False
        self._handle = 0  # native communicator address (CUDA backend), for torch.ops.b200ar
        self._peer_ptrs: List[int] = []
        self._ws_ptr = 0
        self.nvls = None
        self._fast = None  # bound Comm.all_reduce_auto once the CUDA communicator exists

        # Slot capacity: two-shot of max_size, or one-shot push of push_max_size.
        cap = max(
            _C.variant_slot_bytes(sel.VARIANTS["twoshot"], self.cfg.max_size, self.world),
            _C.variant_slot_bytes(sel.VARIANTS["twoshot_push"], self.cfg.max_size, self.world),
            _C.variant_slot_bytes(sel.VARIANTS["oneshot_push"], self.cfg.push_max_size, self.world),
            _C.variant_slot_bytes(sel.VARIANTS["oneshot_pull"], self.cfg.max_size, self.world),
            4096,
        )
        self.slot_capacity = (cap + 255) // 256 * 256

        if self.device.type == "cpu":
            self._init_cpu()
        else:
            self._init_cuda()
        if self.device.type == "cuda" and self.world > 1 and self.cfg.enable_nvls:
            self._init_nvls()
        self.set_selector(sel.load_table(self.world, self.cfg.selector_path or None))

    # ------------------------------------------------------------------ setup
    @property
    def handle(self) -> int:
        """Native communicator handle for the ``torch.ops.b200ar`` operators
        (0 for the CPU backend or after ``close()``)."""
        return self._handle

    def _init_cpu(self) -> None:
        token = [uuid.uuid4().hex[:12] if self.rank == 0 else None]
        dist.broadcast_object_list(token, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                                   group=self.group)
        self.lamport_capacity = (min(self.cfg.lamport_max_size, self.cfg.max_size) + 15) // 16 * 16
        self._shm = _C.ShmComm(f"/b200ar-{token[0]}", self.rank, self.world, self.slot_capacity,
                               self.lamport_capacity if self.world > 1 else 0)
        names: List[Optional[str]] = [None] * self.world
        dist.all_gather_object(names, self._shm.segment_name, group=self.group)
        self._shm.connect(names)
        self._shm.set_timeout_ms(self.cfg.timeout_ms)
        dist.barrier(group=self.group)
        self._comm = None

    def _init_cuda(self) -> None:
        self._shm = None
        with torch.cuda.device(self.device):
            self.lamport_capacity = (min(self.cfg.lamport_max_size, self.cfg.max_size) + 15) // 16 * 16
            ws_bytes = _C.workspace_bytes(self.slot_capacity) + _C.lamport_bytes(self.lamport_capacity, self.world)
            self._ws_ptr = _C.ipc_malloc(ws_bytes)
            handle = _C.ipc_get_handle(self._ws_ptr)
            handles: List[Optional[bytes]] = [None] * self.world
            dist.all_gather_object(handles, handle, group=self.group)
            ptrs = []
            for i, h in enumerate(handles):
                ptrs.append(self._ws_ptr if i == self.rank else int(_C.ipc_open_handle(h)))
            self._peer_ptrs = ptrs
            self._rank_data = torch.empty(self.cfg.rank_data_bytes, dtype=torch.uint8, device=self.device)
            self._comm = _C.Comm(ptrs, self._rank_data, self.rank)
            self._handle = int(self._comm.ptr)
            sig = int(_C.SIGNAL_BYTES)
            self._comm.register_slots(
                [p + sig for p in ptrs], [p + sig + self.slot_capacity for p in ptrs], self.slot_capacity
            )
            if self.world > 1 and self.lamport_capacity > 0:
                lam = _C.workspace_bytes(self.slot_capacity)
                self._comm.register_lamport([p + lam for p in ptrs], self.lamport_capacity)
            self._comm.set_timeout_ns(int(self.cfg.timeout_ms) * 1_000_000)
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        logger.info("rank %d: workspace %d bytes, slot capacity %d", self.rank, ws_bytes, self.slot_capacity)

    def _init_nvls(self) -> None:
        """Creates the NVLS multicast buffer (collective). Any failure on any
        rank disables NVLS on every rank; the other variants stay available."""
        from .nvls import register, setup_multicast

        self.nvls = setup_multicast(self.group, self.rank, self.world, self.device, self.cfg.max_size)
        if self.nvls is not None:
            self._comm.set_nvls(self.nvls)
            register(self)

    def _release_nvls(self) -> None:
        """Waits for this device, detaches and frees the multicast buffer."""
        if self.nvls is None:
            return
        from .nvls import unregister

        torch.cuda.synchronize(self.device)
        if self._comm is not None:
            self._comm.set_nvls(None)
        self.nvls = None  # NvlsBuffer destructor unmaps, unbinds and releases
        unregister(self)

    # -------------------------------------------------------------- selection
    def set_selector(self, entries) -> None:
        self.selector = list(entries)
        if self._comm is not None:
            self._comm.set_selector(sel.to_native(self.selector))
            self._fast = self._comm.all_reduce_auto if self.cfg.variant == "auto" else None

    def plan(self, nbytes: int, variant="auto", ctas: int = 0):
        """(variant name, ctas, threads) that a message of ``nbytes`` would use."""
        if self._comm is None:
            return ("cpu", ctas, 0)
        v, c, t = self._comm.plan(int(nbytes), sel.variant_id(variant), int(ctas))
        return (sel.VARIANT_NAMES[v], c, t)

    def supports(self, t: torch.Tensor) -> bool:
        """True when ``t`` can be served by the custom kernels (else NCCL)."""
        nbytes = t.numel() * t.element_size()
        return (
            t.dtype in (torch.float32, torch.float16, torch.bfloat16)
            and nbytes % 16 == 0
            and t.data_ptr() % 16 == 0
            and t.is_contiguous()
        )

    # --------------------------------------------- serving-engine interface
    @property
    def disabled(self) -> bool:
        return self.closed

    def should_custom_ar(self, inp: torch.Tensor) -> bool:
        """True when b200ar's own kernels serve ``inp`` (the interface of the
        custom all-reduce wrappers in vLLM / SGLang): a supported dtype and
        layout, within ``max_size``, and below the measured NCCL crossover."""
        if self.closed or not self.supports(inp):
            return False
        nbytes = inp.numel() * inp.element_size()
        if nbytes > self.cfg.max_size:
            return False
        return self.plan(nbytes)[0] != "nccl"

    def custom_all_reduce(self, inp: torch.Tensor) -> Optional[torch.Tensor]:
        """Out-of-place all-reduce if ``should_custom_ar(inp)``, else None (the
        caller then uses its NCCL path), as in those wrappers."""
        if not self.should_custom_ar(inp):
            return None
        return self.all_reduce(inp)

    # ------------------------------------------------------------ collectives
    def all_reduce(self, inp: torch.Tensor, out: Optional[torch.Tensor] = None, variant="auto",
                   ctas: int = 0) -> torch.Tensor:
        """Returns the elementwise sum of ``inp`` over all ranks (``out`` may alias ``inp``).

        Contiguous float32/float16/bfloat16 tensors of a multiple of 16 bytes
        on a 16-byte boundary run on the b200ar kernels (or NCCL above the
        measured crossover). Other tensors go to NCCL when an NCCL group is
        available, else through a zero-padded contiguous copy."""
        if out is None:
            out = torch.empty_like(inp)
        fast = self._fast
        if fast is not None and variant == "auto" and not ctas and not torch.compiler.is_compiling():
            # Lean eager path: dtype/layout/alignment checks, plan and launch in one native call.
            if fast(inp, out):
                return out
        if self.closed:
            raise RuntimeError("communicator is closed")
        v = sel.variant_id(variant if variant != "auto" else self.cfg.variant)
        if torch.compiler.is_compiling() and self._handle:
            # Traced by torch.compile: one dispatcher op, no host-side fallback
            # (messages above the NCCL crossover run the two-shot kernel).
            torch.ops.b200ar.all_reduce(self._handle, inp, out, v, int(ctas))
            return out
        if not (self.supports(inp) and self.supports(out)):
            if self._comm is not None and self.nccl_group is not None:
                return self._nccl(inp, out)
            return self._staged(inp, out, variant, ctas)
        if self._comm is None:
            # The CPU emulation implements the slot variants and the Lamport one-shot.
            cpu_ok = (sel.VARIANTS["oneshot_push"], sel.VARIANTS["oneshot_pull"], sel.VARIANTS["twoshot"],
                      sel.VARIANTS["twoshot_push"], sel.VARIANTS["lamport"])
            if v not in cpu_ok or (v == sel.VARIANTS["lamport"]
                                   and inp.numel() * inp.element_size() > self.lamport_capacity):
                v = sel.VARIANTS["auto"]
            self._shm.all_reduce(inp, out, v, ctas)
            return out
        if v == sel.VARIANTS["nccl"]:
            return self._nccl(inp, out)
        launched = self._comm.all_reduce(inp, out, v, ctas)
        if launched == sel.VARIANTS["nccl"]:
            # Above the measured crossover (which was measured on this same
            # out-of-place NCCL path) or beyond the slot capacity.
            return self._nccl(inp, out)
        return out

    def all_reduce_residual_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
                                    eps: float = 1e-5, out: Optional[torch.Tensor] = None,
                                    residual_out: Optional[torch.Tensor] = None, variant="auto", ctas: int = 0):
        """Fused TP decode epilogue: ``z = all_reduce(x) + residual``,
        ``out = RMSNorm(z) * gamma``. Returns ``(out, z)``; ``residual_out`` may
        alias ``residual`` (in-place residual update) and ``out`` may alias ``x``."""
        if out is None:
            out = torch.empty_like(x)
        if residual_out is None:
            residual_out = torch.empty_like(residual)
        if torch.compiler.is_compiling() and self._handle:
            torch.ops.b200ar.all_reduce_residual_rmsnorm(self._handle, x, residual, gamma, float(eps), out,
                                                         residual_out, sel.variant_id(variant), int(ctas))
            return out, residual_out
        if self._comm is None:
            z = self.all_reduce(x.float().contiguous()) + residual.float()
            zb = z.to(residual.dtype)
            zf = zb.float()
            y = zf * torch.rsqrt(zf.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()
            residual_out.copy_(zb)
            out.copy_(y.to(out.dtype))
            return out, residual_out
        self._comm.ar_rmsnorm(x, residual, gamma, out, residual_out, float(eps), sel.variant_id(variant), int(ctas))
        return out, residual_out

    def linear_all_reduce(self, x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                          fused: bool = True) -> torch.Tensor:
        """Row-parallel linear: ``sum over ranks of x_r @ w_r.T`` (bf16).

        With ``fused`` (default) one persistent tcgen05 kernel computes the
        partial tiles and pushes each one to its owner rank from the epilogue
        (reduce-scatter), then the owners publish the reduced tiles
        (all-gather). Shapes the fused kernel cannot serve fall back to the
        tcgen05 GEMM followed by ``all_reduce``."""
        from ..ops.gemm import error_word, linear

        m, n = x.shape[0], w.shape[0]
        if out is None:
            out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
        # Below ~512 rows the 128x256 tiles leave most SMs idle; the split-K
        # decode GEMM followed by the (Lamport) all-reduce is faster there.
        if fused and m < 512:
            fused = False
        if fused and self._comm is not None and self.world > 1 and self._comm.gemm_ar_supported(m, n):
            self._comm.gemm_allreduce(x.contiguous(), w, out, error_word(x.device))
            return out
        partial = linear(x, w)
        return self.all_reduce(partial, out=out)

    def all_gather_linear(self, x_shard: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                          fused: bool = True) -> torch.Tensor:
        """Column-parallel linear on sequence-sharded input:
        ``concat over ranks of x_shard (rows) @ w.T``. Fused, the GEMM's TMA
        producer reads every shard straight from its owner over NVLink; other
        shapes fall back to an all-gather followed by the tcgen05 GEMM."""
        from ..ops.gemm import error_word, linear

        rows, k = x_shard.shape
        if out is None:
            out = torch.empty(rows * self.world, w.shape[0], dtype=torch.bfloat16, device=x_shard.device)
        if fused and self._comm is not None and self._comm.ag_gemm_supported(rows, k):
            self._comm.ag_gemm(x_shard.contiguous(), w, out, error_word(x_shard.device))
            return out
        full = torch.empty(rows * self.world, k, dtype=x_shard.dtype, device=x_shard.device)
        if self.world > 1 and self._comm is None:  # CPU backend: gather over the bootstrap group
            parts = [torch.empty_like(x_shard) for _ in range(self.world)]
            dist.all_gather(parts, x_shard.contiguous(), group=self.group)
            torch.cat(parts, dim=0, out=full)
        elif self.world > 1:
            dist.all_gather_into_tensor(full, x_shard.contiguous(), group=self.nccl_group)
        else:
            full.copy_(x_shard)
        return linear(full, w, out=out)

    def _staged(self, inp: torch.Tensor, out: torch.Tensor, variant, ctas: int) -> torch.Tensor:
        """Serves a tensor the kernels cannot take as it is (size not a
        multiple of 16 bytes, misaligned or strided) through a zero-padded
        contiguous copy when no NCCL group is available."""
        if inp.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise TypeError(f"b200ar all-reduce supports float32, float16 and bfloat16, not {inp.dtype}")
        if out.dtype != inp.dtype or out.numel() != inp.numel():
            raise ValueError("input and output must have the same dtype and number of elements")
        n = inp.numel()
        per16 = 16 // inp.element_size()
        buf = torch.zeros((n + per16 - 1) // per16 * per16, dtype=inp.dtype, device=inp.device)
        buf[:n].copy_(inp.reshape(-1))
        res = self.all_reduce(buf, variant=variant, ctas=ctas)
        out.copy_(res[:n].reshape(out.shape))
        return out

    def _nccl(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if self.nccl_group is None:
            raise RuntimeError(
                "message cannot be served by the custom kernels (size/alignment/capacity) and no NCCL group "
                "was given for the fallback"
            )
        n = inp.numel()
        if (out.data_ptr() != inp.data_ptr() and self.world > 1 and n % self.world == 0 and inp.is_contiguous()
                and out.is_contiguous()):
            # Out of place without the extra copy: reduce-scatter into this
            # rank's shard of `out`, then an in-place all-gather of the shards.
            shard = out.view(-1).narrow(0, self.rank * (n // self.world), n // self.world)
            dist.reduce_scatter_tensor(shard, inp.view(-1), group=self.nccl_group)
            dist.all_gather_into_tensor(out.view(-1), shard, group=self.nccl_group)
            return out
        if out.data_ptr() != inp.data_ptr():
            out.copy_(inp)
        dist.all_reduce(out, group=self.nccl_group)
        return out

    # ----------------------------------------------- registered buffers / graphs
    def register_buffer(self, t: torch.Tensor) -> None:
        """Registers ``t`` (allocated by ``cudaMalloc``-backed memory, e.g.
        ``b200ar.ipc.CudaIPC().malloc``) for the zero-copy variant: collective."""
        ptrs = exchange_ptr(t.data_ptr(), self.group)
        self._comm.register_buffer(ptrs)

    @contextlib.contextmanager
    def capture(self):
        """Context for capturing a CUDA graph that uses the zero-copy
        ``variant="registered"`` path: on exit, the input addresses recorded
        during capture are exchanged and registered (collective). Calls that use
        the slot variants need no registration and work in graphs as they are."""
        try:
            yield self
        finally:
            self.register_graph_buffers()

    def register_graph_buffers(self) -> None:
        if self._comm is None:
            return
        try:
            handles, offsets = self._comm.graph_buffer_meta()
        except RuntimeError as e:
            from ..ipc import allocator_blocks_ipc

            why = allocator_blocks_ipc()
            if why is None:
                raise
            raise RuntimeError(f"cannot export the inputs captured for variant='registered' while {why} is set; "
                               "use the slot variants in graphs (no registration needed) or unset it") from e
        meta: List[Optional[tuple]] = [None] * self.world
        dist.all_gather_object(meta, (handles, offsets), group=self.group)
        self._comm.register_graph_buffers([m[0] for m in meta], [m[1] for m in meta])

    # ------------------------------------------------------- status and reset
    def check(self) -> None:
        """Raises ``CommTimeoutError`` if a kernel reported a barrier timeout."""
        if self._comm is not None:
            self._comm.check()

    def status(self) -> dict:
        return self._comm.status() if self._comm is not None else {"code": self._shm.status_code()}

    def reset(self) -> None:
        """Collective recovery after a timeout: every rank zeroes its signal
        block between two barriers of the bootstrap group."""
        if self._comm is not None:
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        if self._comm is not None:
            self._comm.reset()
        else:
            self._shm.reset()
        dist.barrier(group=self.group)

    @property
    def launches(self) -> int:
        """Number of kernels launched by this communicator so far."""
        return self._comm.launches if self._comm is not None else 0

    def close(self) -> None:
        """Collective teardown: waits until no peer can still touch this rank's
        workspace (device sync + group barrier), then unmaps and frees it."""
        if self.closed:
            return
        self.closed = True
        self._fast = None
        if self._comm is not None:
            torch.cuda.synchronize(self.device)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        self._release_nvls()
        if self._comm is not None:
            del self._comm
            self._comm = None
            self._handle = 0
            for i, p in enumerate(self._peer_ptrs):
                if i != self.rank:
                    _C.ipc_close_handle(p)
            if self._ws_ptr:
                _C.ipc_free(self._ws_ptr)
                self._ws_ptr = 0
        self._shm = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def exchange_ptr(ptr: int, group=None) -> List[int]:
    from ..ipc import exchange_buffers

    return exchange_buffers(ptr, group)
