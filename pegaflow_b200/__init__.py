"""B200-native KV-cache block transfer path with PegaFlow's engine API.

Public surface (mirrors the reference's ``pegaflow.pegaflow`` module):
  PegaEngine, PyLoadState        in-process engine + shm load flag
  Executor, Layout, SaveSpec ... transfer executor (C ABI pf_executor_*)

The native library is loaded on first use of any of these names, so
``pegaflow_b200.build`` can run before the library exists. A missing or
broken library raises ImportError at that first use; there is no fallback.
"""

import importlib

_EXPORTS = {
    "PegaEngine": ".engine",
    "PyLoadState": ".engine",
    "EngineRpcClient": ".client",
    "CudaIPCWrapper": ".ipc",
    "PegaError": "._native",
    "LIB_PATH": "._native",
    "Executor": ".transfer",
    "Layout": ".transfer",
    "LoadSpec": ".transfer",
    "SaveSpec": ".transfer",
    "P2PSpec": ".transfer",
    "PinnedBuffer": ".transfer",
    "refcopy_save": ".transfer",
    "refcopy_load": ".transfer",
    "segment_offset": ".transfer",
    "validate": ".transfer",
}

__all__ = sorted(_EXPORTS)


def __getattr__(name):
    if name in _EXPORTS:
        value = getattr(importlib.import_module(_EXPORTS[name], __name__), name)
        globals()[name] = value
        return value
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
