"""Reference-compatible op set.

Exactly the eight functions that ``pcie_allreduce`` exports
(pcie_allreduce/__init__.py:22-29, pcie_allreduce.cu:596-606), with the same
argument lists, so code written against the reference or against
``sgl_kernel.allreduce`` switches by changing the import::

    import b200ar.compat as pcie_allreduce

Semantics are those of the reference, with these fixes:

* ``all_reduce`` with double buffers registered (``register_pcie_buffers``)
  picks one-shot push, two-shot or one-shot pull by message size and slot
  capacity, and it keeps using the double buffers inside CUDA graphs (the slot
  is chosen on the device), so ``get_graph_buffer_ipc_meta`` then returns empty
  lists and ``register_graph_buffers`` is a no-op.
* A message that does not fit the registered capacity raises instead of
  overflowing it (the reference's pull path did not check, cu:420-446).
* ``buf_capacity=0`` means "use the allocation size" rather than "pull only".
* The zero-copy registered path has an end barrier (no write-after-read race).
"""

from ._native import _C
from .ipc import allocator_blocks_ipc

init_custom_ar = _C.init_custom_ar
all_reduce = _C.all_reduce
dispose = _C.dispose
meta_size = _C.meta_size
register_buffer = _C.register_buffer
register_pcie_buffers = _C.register_pcie_buffers
register_graph_buffers = _C.register_graph_buffers



def get_graph_buffer_ipc_meta(fa: int):
    """IPC handles (as byte lists) and offsets of the inputs captured since the
    last registration. The error names the allocator setting when one makes
    the captured tensors non-exportable."""
    try:
        return _C.get_graph_buffer_ipc_meta(fa)
    except RuntimeError as e:
        why = allocator_blocks_ipc()
        if why is None:
            raise
        raise RuntimeError(f"cannot export the captured all-reduce inputs over CUDA IPC while {why} is set; "
                           "unset it or capture with registered double buffers (register_pcie_buffers)") from e


__all__ = [
    "init_custom_ar",
    "all_reduce",
    "dispose",
    "meta_size",
    "register_buffer",
    "register_pcie_buffers",
    "get_graph_buffer_ipc_meta",
    "register_graph_buffers",
]
