"""Runtime configuration of b200ar.

The reference hard-codes its knobs (kMaxBlocks=36 and 512 threads,
pcie_allreduce.cu:46 and :401; buffer sizes in each script). Here they live in
one dataclass whose defaults can be overridden by ``B200AR_*`` environment
variables or by keyword arguments.
"""

from __future__ import annotations

import dataclasses
import os
from typing import Optional


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


@dataclasses.dataclass
class Config:
    # Largest message (bytes) served by the custom kernels; larger ones go to NCCL.
    max_size: int = dataclasses.field(default_factory=lambda: _env_int("B200AR_MAX_SIZE", 64 << 20))
    # Largest message (bytes) for which the one-shot push variant is allowed.
    push_max_size: int = dataclasses.field(default_factory=lambda: _env_int("B200AR_PUSH_MAX_SIZE", 1 << 20))
    # Largest message (bytes) for the barrier-free one-shot Lamport variant.
    lamport_max_size: int = dataclasses.field(default_factory=lambda: _env_int("B200AR_LAMPORT_MAX_SIZE", 4 << 20))
    # Barrier wait limit before a kernel reports a timeout.
    timeout_ms: int = dataclasses.field(default_factory=lambda: _env_int("B200AR_TIMEOUT_MS", 10000))
    # Force a variant for every call ("auto", "oneshot_push", "oneshot_pull", "twoshot", "nvls", "nccl").
    variant: str = dataclasses.field(default_factory=lambda: os.environ.get("B200AR_VARIANT", "auto"))
    # Path of a measured selector table (JSON); empty = packaged default.
    selector_path: str = dataclasses.field(default_factory=lambda: os.environ.get("B200AR_SELECTOR", ""))
    # Try NVLS (multimem) when the devices support multicast (opt-in: B200AR_NVLS=1).
    enable_nvls: bool = dataclasses.field(default_factory=lambda: os.environ.get("B200AR_NVLS", "0") == "1")
    # Bytes of the device arena holding peer-pointer records for registered buffers.
    rank_data_bytes: int = dataclasses.field(default_factory=lambda: _env_int("B200AR_RANK_DATA_BYTES", 8 << 20))

    def replace(self, **kw) -> "Config":
        return dataclasses.replace(self, **kw)


def default_config(overrides: Optional[dict] = None) -> Config:
    cfg = Config()
    if overrides:
        cfg = cfg.replace(**{k: v for k, v in overrides.items() if v is not None})
    return cfg
