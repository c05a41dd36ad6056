"""servoflow_b200 — B200-native (sm_100a) attention path for servoflow's
RDT-1B runtime.

The product is libsfb200.so (servoflow_b200/csrc, C ABI in include/sfb200.h).
This package builds it and exposes a thin Python mirror of the reference's
IBackend ops for tests and benchmarks.
"""
from ._capi import LIB_PATH, SfbError, lib, status_string  # noqa: F401

__version__ = "0.1.0"


def backend(device: int = 0):
    from .backend import B200Backend
    return B200Backend(device)
