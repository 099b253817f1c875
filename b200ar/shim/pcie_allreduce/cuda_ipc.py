"""``pcie_allreduce.cuda_ipc`` served by b200ar (b200ar.ipc)."""

from b200ar.ipc import CudaIPC, cudaIpcMemHandle_t  # noqa: F401
