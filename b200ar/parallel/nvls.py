"""Collective set-up of the NVLS (NVLink SHARP) multicast buffer.

Rank 0 creates the multicast object and exports it as a POSIX file
descriptor; the descriptor travels to the other ranks of this node over an
abstract Unix-domain socket (``SCM_RIGHTS``); every rank adds its device, and
after a barrier binds its own physical memory and maps both the multicast and
the local view. Returns ``None`` on every rank if any rank cannot take part
(no multicast support, driver refusal, ...).
"""

from __future__ import annotations

import atexit
import os
import socket
import time
import uuid
from typing import Optional

import torch.distributed as dist

from .._native import _C
from ..log import logger


# Communicators holding a multicast buffer. A process that ends with device
# memory still bound to a multicast object can fault the peers' GPUs, so the
# buffers are unbound at interpreter exit even if close() was never called.
_LIVE = []


def register(comm) -> None:
    _LIVE.append(comm)


def unregister(comm) -> None:
    if comm in _LIVE:
        _LIVE.remove(comm)


@atexit.register
def _release_all() -> None:
    for comm in list(_LIVE):
        try:
            comm._release_nvls()
        except Exception:  # noqa: BLE001 - interpreter teardown
            pass
    _LIVE.clear()


def _all_ok(flag: bool, group) -> bool:
    flags = [None] * dist.get_world_size(group)
    dist.all_gather_object(flags, bool(flag), group=group)
    return all(flags)


def _share_fd(fd: Optional[int], rank: int, world: int, group) -> int:
    """Sends rank 0's ``fd`` to every other rank; returns the local descriptor."""
    token = [f"b200ar-nvls-{uuid.uuid4().hex}" if rank == 0 else None]
    dist.broadcast_object_list(token, src=dist.get_global_rank(group, 0) if group else 0, group=group)
    addr = "\0" + token[0]
    if rank == 0:
        srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        srv.bind(addr)
        srv.listen(world)
        dist.barrier(group=group)
        for _ in range(world - 1):
            conn, _ = srv.accept()
            with conn:
                socket.send_fds(conn, [b"m"], [fd])
        srv.close()
        dist.barrier(group=group)
        return fd
    dist.barrier(group=group)
    cli = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    for _ in range(100):
        try:
            cli.connect(addr)
            break
        except OSError:
            time.sleep(0.05)
    _, fds, _, _ = socket.recv_fds(cli, 1, 1)
    cli.close()
    dist.barrier(group=group)
    return fds[0]


def setup_multicast(group, rank: int, world: int, device, nbytes: int):
    dev = device.index if device.index is not None else 0
    ok = _C.NvlsBuffer.supported(dev)
    if not _all_ok(ok, group):
        logger.info("NVLS disabled: multicast not supported on every device")
        return None
    buf = None
    fd = None
    err = None
    try:
        buf = _C.NvlsBuffer(dev, world, int(nbytes))
        if rank == 0:
            fd = buf.create_and_export()
    except Exception as e:  # noqa: BLE001 - reported collectively
        err = e
    if not _all_ok(err is None, group):
        logger.warning("NVLS disabled: multicast object creation failed (%s)", err)
        return None
    try:
        fd = _share_fd(fd, rank, world, group)
        if rank != 0:
            buf.import_handle(fd)
        buf.add_device()
    except Exception as e:  # noqa: BLE001
        err = e
    finally:
        if fd is not None:
            os.close(fd)
    if not _all_ok(err is None, group):
        logger.warning("NVLS disabled: multicast import/add failed (%s)", err)
        return None
    try:
        buf.bind_and_map()
    except Exception as e:  # noqa: BLE001
        err = e
    if not _all_ok(err is None, group):
        logger.warning("NVLS disabled: multicast bind/map failed (%s)", err)
        return None
    logger.info("rank %d: NVLS buffer of %d bytes mapped", rank, buf.bytes)
    return buf
