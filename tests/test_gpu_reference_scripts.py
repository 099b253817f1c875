"""The reference's own multi-GPU scripts, unmodified, running on b200ar.

``b200ar.shim`` serves the reference's import names (``pcie_allreduce``,
``pcie_allreduce.cuda_ipc``, ``cuda_ipc``), so a program written against the
reference runs on b200ar when the shim directory is first on ``PYTHONPATH``.
This test runs the reference's smoke test (test_pcie_ar.py) and its eleven
stress scenarios (stress_test.py) that way, on every visible GPU (up to 8).

The scripts are taken from the reference checkout installed beside the
reference package (``baseline/_ref/scripts/``, not part of this repository);
the test skips when they are absent. They sit in a directory without a
``pcie_allreduce`` package, so the import resolves to the shim.
"""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SCRIPTS = os.path.join(ROOT, "baseline", "_ref", "scripts")
NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0
if NGPU < 2:
    pytest.skip("needs at least two GPUs", allow_module_level=True)
WORLD = min(NGPU, 8) // 2 * 2  # the reference accepts even world sizes only


def _run(script, marker, timeout):
    path = os.path.join(SCRIPTS, script)
    if not os.path.exists(path):
        pytest.skip(f"reference script {script} is not installed under baseline/_ref/scripts")
    import b200ar.shim

    # No reference package next to the script: `import pcie_allreduce` finds the shim.
    assert not os.path.exists(os.path.join(SCRIPTS, "pcie_allreduce"))

    env = dict(os.environ, PYTHONPATH=os.pathsep.join([b200ar.shim.shim_path(), ROOT]), NCCL_NVLS_ENABLE="0")
    res = subprocess.run([sys.executable, path, str(WORLD)], cwd=SCRIPTS, env=env, capture_output=True, text=True,
                         timeout=timeout)
    out = res.stdout + res.stderr
    assert res.returncode == 0, out[-6000:]
    assert marker in res.stdout, out[-6000:]
    assert "FAIL" not in res.stdout, out[-6000:]
    return res.stdout


def test_reference_smoke_script_on_shim():
    _run("test_pcie_ar.py", "ALL TESTS PASSED", 900)


def test_reference_stress_script_on_shim():
    _run("stress_test.py", "ALL STRESS TESTS PASSED", 1800)
