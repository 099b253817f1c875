"""Loads the in-tree native library ``b200ar._C`` (built by ``setup.py build_ext --inplace``).

If the shared object is missing, it is built once (under a file lock) unless
``B200AR_NO_BUILD=1``. On a machine with a GPU a missing or broken extension is
an error: b200ar never falls back silently to a pure-PyTorch path.

With ``B200AR_CHECKS=1`` the checked debug build ``b200ar._C_checked`` is
loaded (and built) instead: its kernels verify access ranges and barrier
epochs on the device and report violations through the status record.
"""

from __future__ import annotations

import fcntl
import importlib
import os
import subprocess
import sys

import torch  # noqa: F401 - loads libc10/libtorch before the extension

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_inplace(verbose: bool = False) -> None:
    """Compiles every native source for sm_100a into ``b200ar/_C*.so`` (the
    checked build when ``B200AR_CHECKS=1`` is in the environment)."""
    os.makedirs(os.path.join(_ROOT, "build"), exist_ok=True)
    lock_path = os.path.join(_ROOT, "build", ".b200ar_build.lock")
    with open(lock_path, "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        env = dict(os.environ)
        env.setdefault("MAX_JOBS", str(max(1, min(16, os.cpu_count() or 1))))
        cmd = [sys.executable, "setup.py", "build_ext", "--inplace"]
        res = subprocess.run(cmd, cwd=_ROOT, env=env, capture_output=not verbose, text=True)
        if res.returncode != 0:
            tail = (res.stdout or "")[-4000:] + (res.stderr or "")[-4000:]
            raise RuntimeError(f"building b200ar._C failed:\n{tail}")


def module_name() -> str:
    return "b200ar._C_checked" if os.environ.get("B200AR_CHECKS") == "1" else "b200ar._C"


def load():
    name = module_name()
    try:
        return importlib.import_module(name)
    except ImportError:
        if os.environ.get("B200AR_NO_BUILD") == "1":
            raise
    build_inplace()
    importlib.invalidate_caches()
    return importlib.import_module(name)


_C = load()
