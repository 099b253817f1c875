"""Communication layer: the custom all-reduce communicator, its selector and
the NVLS (multicast) path."""

from .comm import CommTimeoutError, CustomAllreduce  # noqa: F401
from . import selector  # noqa: F401
