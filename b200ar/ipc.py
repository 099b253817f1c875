"""CUDA IPC buffer helpers.

Drop-in for the reference's ``cuda_ipc.CudaIPC`` (pcie_allreduce/cuda_ipc.py:26-92):
same method names and return types (``ctypes.c_void_p`` pointers and a 64-byte
``cudaIpcMemHandle_t`` structure), backed by the native library instead of a
ctypes scan of ``/proc/self/maps``. Additions: ``ipc_close_handle`` (the
reference never closed handles), reference-counted opening (opening the same
handle twice returns the same mapping), and helpers to exchange handles over a
``torch.distributed`` group.
"""

from __future__ import annotations

import ctypes
import os
from typing import List, Optional

import torch.distributed as dist

from ._native import _C

HANDLE_BYTES = int(_C.IPC_HANDLE_BYTES)


class cudaIpcMemHandle_t(ctypes.Structure):  # noqa: N801 - CUDA's type name
    _fields_ = [("internal", ctypes.c_byte * HANDLE_BYTES)]

    def to_bytes(self) -> bytes:
        return bytes(bytearray(self.internal))

    @classmethod
    def from_bytes(cls, b: bytes) -> "cudaIpcMemHandle_t":
        if len(b) != HANDLE_BYTES:
            raise ValueError(f"IPC handle must be {HANDLE_BYTES} bytes, got {len(b)}")
        h = cls()
        ctypes.memmove(ctypes.addressof(h), b, HANDLE_BYTES)
        return h

    def __reduce__(self):  # picklable for all_gather_object
        return (cudaIpcMemHandle_t.from_bytes, (self.to_bytes(),))


def _as_int(ptr) -> int:
    return int(ptr.value if isinstance(ptr, ctypes.c_void_p) else ptr)


class CudaIPC:
    """cudaMalloc / cudaFree / cudaMemset / cudaIpc{Get,Open,Close}MemHandle."""

    def __init__(self, so_file: Optional[str] = None):
        # so_file is accepted for signature compatibility; the native library is used.
        del so_file

    def malloc(self, size: int) -> ctypes.c_void_p:
        return ctypes.c_void_p(_C.ipc_malloc(int(size)))

    def free(self, ptr) -> None:
        _C.ipc_free(_as_int(ptr))

    def memset(self, ptr, value: int, count: int) -> None:
        _C.ipc_memset(_as_int(ptr), int(value), int(count))

    def ipc_get_handle(self, ptr) -> cudaIpcMemHandle_t:
        return cudaIpcMemHandle_t.from_bytes(export_handle(_as_int(ptr)))

    def ipc_open_handle(self, handle) -> ctypes.c_void_p:
        raw = handle.to_bytes() if isinstance(handle, cudaIpcMemHandle_t) else bytes(handle)
        return ctypes.c_void_p(_C.ipc_open_handle(raw))

    def ipc_close_handle(self, ptr) -> None:
        _C.ipc_close_handle(_as_int(ptr))


def allocator_blocks_ipc() -> Optional[str]:
    """Names the PyTorch allocator setting under which tensor memory cannot be
    exported with ``cudaIpcGetMemHandle`` (``expandable_segments`` maps memory
    with the virtual-memory API; the ``cudaMallocAsync`` backend allocates from
    a stream-ordered pool), or None."""
    for var in ("PYTORCH_CUDA_ALLOC_CONF", "PYTORCH_ALLOC_CONF"):
        for item in os.environ.get(var, "").replace(";", ",").split(","):
            key, _, value = item.partition(":")
            key, value = key.strip().lower(), value.strip().lower()
            if key == "expandable_segments" and value == "true":
                return f"{var}=expandable_segments:True"
            if key == "backend" and value == "cudamallocasync":
                return f"{var}=backend:cudaMallocAsync"
    return None


def export_handle(ptr: int) -> bytes:
    """``cudaIpcGetMemHandle`` of the allocation holding ``ptr``. When the
    export fails under an allocator setting that makes tensor memory
    non-exportable, the error names that setting and the way out."""
    try:
        return _C.ipc_get_handle(int(ptr))
    except RuntimeError as e:
        why = allocator_blocks_ipc()
        if why is None:
            raise
        raise RuntimeError(
            f"cannot export address {int(ptr):#x} over CUDA IPC while {why} is set: that allocator setting "
            "gives memory cudaIpcGetMemHandle cannot export. Allocate registered buffers with "
            "b200ar.ipc.CudaIPC().malloc (plain cudaMalloc), or unset the setting."
        ) from e


def exchange_buffers(ptr: int, group=None) -> List[int]:
    """All-gathers the IPC handle of this rank's allocation ``ptr`` and returns
    every rank's pointer as mapped in this process (own pointer at own rank)."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    handle = export_handle(ptr)
    handles: List[Optional[bytes]] = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    out = []
    for i, h in enumerate(handles):
        out.append(int(ptr) if i == rank else int(_C.ipc_open_handle(h)))
    return out


def close_buffers(ptrs: List[int], rank: int) -> None:
    for i, p in enumerate(ptrs):
        if i != rank:
            _C.ipc_close_handle(int(p))
