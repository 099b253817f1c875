"""Drop-in import names of the reference library, served by b200ar.

The directory of this package holds ``pcie_allreduce/`` (the eight ops of
``pcie_allreduce/__init__.py:22-29`` and its ``cuda_ipc`` module) and a
top-level ``cuda_ipc`` module (imported that way by the reference's
``stress_test.py:35``). With ``shim_path()`` first on ``PYTHONPATH``, code
written against ``pcie_allreduce`` runs on b200ar without edits::

    PYTHONPATH=$(python -c "import b200ar.shim as s; print(s.shim_path())") python test_pcie_ar.py 2
"""

import os


def shim_path() -> str:
    """Directory to put first on ``sys.path`` / ``PYTHONPATH``."""
    return os.path.dirname(os.path.abspath(__file__))
