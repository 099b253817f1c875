"""``pcie_allreduce`` served by b200ar: the same eight ops (b200ar.compat)."""

from b200ar.compat import (  # noqa: F401
    __all__,
    all_reduce,
    dispose,
    get_graph_buffer_ipc_meta,
    init_custom_ar,
    meta_size,
    register_buffer,
    register_graph_buffers,
    register_pcie_buffers,
)
