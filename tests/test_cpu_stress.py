"""The stress suite (the reference's scenarios t1-t9 plus the random-size run)
on two CPU ranks through torchrun: gloo bootstrap, shared-memory data plane."""

import os
import subprocess
import sys

from dist_util import free_port

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_stress_suite_cpu_two_ranks():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), os.path.join(ROOT, "bench", "stress.py"),
           "--device", "cpu", "--random-iters", "300", "--max-random-bytes", str(1 << 20), "--check-every", "50"]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    out = res.stdout + res.stderr
    assert res.returncode == 0, out[-4000:]
    assert "ALL STRESS TESTS PASSED" in res.stdout, out[-4000:]
    for name in ("rapid_fire", "unique_values", "back_to_back", "continuous_batching", "random_sizes"):
        assert f"{name}" in res.stdout and "FAIL" not in res.stdout


def test_stress_sync_helpers_do_not_recurse():
    """The GPU branch's sync helper must be the device synchronize itself (a
    helper that called itself once made every GPU scenario fail at its first
    sync); the CPU one must return without waiting."""
    import importlib.util

    import torch

    spec = importlib.util.spec_from_file_location("stress_main", os.path.join(ROOT, "bench", "stress.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.make_sync(True) is torch.cuda.synchronize
    assert mod.make_sync(False)() is None
