"""kbb200 — B200 (sm_100a) fp32 operator library behind the kernelbench-hip
candidate API.

    import kbb200
    y = kbb200.ops.gelu_tanh(x)          # tensor-level API
    kbb200.ext.mingpt_gelu_entry(x, y)   # candidate entry names (EXT.<ENTRY>)

Importing this package loads libkbb200.so (C ABI, include/kbb200.h) and fails
if it has not been built.
"""
from . import _lib, ext, ops  # noqa: F401
from ._lib import LIB, KbError, LIB_PATH  # noqa: F401

__version__ = "0.1.0"


def version() -> int:
    return LIB.kb_version()
