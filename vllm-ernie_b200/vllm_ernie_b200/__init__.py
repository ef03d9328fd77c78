"""B200-native (sm_100a) implementation of the ERNIE 5.5 HCA layer path.

The compute lives in ``lib/libhca_b200.so`` (C ABI: ``include/hca_b200.h``);
this package is the host side: the ctypes loader, torch-facing op wrappers
named after the reference ops they replace, the decode hot path, synthetic
workloads, and the module / backend API the ERNIE 5.5 model code calls.
"""

from . import ops  # noqa: F401
from ._lib import HcaError, lib  # noqa: F401

__version__ = "0.1.0"


def register() -> None:
    """Plugin entry point, idempotent (``src/vllm_ernie/__init__.py:14-31``).
    Loads the kernel library so a missing build fails at registration."""
    lib()
