"""kbb200 — B200 (sm_100a) fp32 operator library behind the kernelbench-hip
candidate API.

    import kbb200
    y = kbb200.ops.gelu_tanh(x)          # tensor-level API
    kbb200.ext.mingpt_gelu_entry(x, y)   # candidate entry names (EXT.<ENTRY>)

The submodules that launch kernels (`ops`, `ext`, `p2p`, `_lib`) load
libkbb200.so (C ABI, include/kbb200.h) when they are first imported, and
`dist` when it first calls a kernel; they fail if it has not been built, and
there is no other implementation to fall back to.  Importing the package
itself, or its pure-host modules (`workloads`, `launch`, `milestone_table`),
loads nothing, so a process that only plans or sweeps work (the CPU
reference timing, the multi-GPU launcher) never maps the library.
"""
from __future__ import annotations

import importlib

__version__ = "0.2.0"

_SUBMODULES = {"_lib", "ops", "ext", "dist", "p2p", "workloads", "launch", "milestone_table"}
_FROM_LIB = {"LIB", "KbError", "LIB_PATH"}


def __getattr__(name: str):
    if name in _SUBMODULES:
        return importlib.import_module(f".{name}", __name__)
    if name in _FROM_LIB:
        return getattr(importlib.import_module("._lib", __name__), name)
    raise AttributeError(f"module 'kbb200' has no attribute {name!r}")


def version() -> int:
    return importlib.import_module("._lib", __name__).LIB.kb_version()
