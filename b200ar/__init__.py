"""b200ar: custom all-reduce and fused tensor-parallel kernels for NVIDIA B200
(sm_100a) over NVLink 5 / NVSwitch.

Public API:
  * ``b200ar.CustomAllreduce``   idiomatic communicator (bootstrap included)
  * ``b200ar.compat``            the reference's eight-op ABI (pcie_allreduce)
  * ``b200ar.ipc.CudaIPC``       CUDA IPC buffer helper (cuda_ipc.CudaIPC)
  * ``b200ar.ops``               fused TP ops (all-reduce + residual + RMSNorm, ...)
  * ``b200ar.models``            TP decoder slice built on the above
"""

from ._native import _C  # noqa: F401
from .config import Config, default_config  # noqa: F401
from .parallel.comm import CommTimeoutError, CustomAllreduce  # noqa: F401

__version__ = "0.1.0"
