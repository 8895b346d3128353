"""B200-native KV-cache block transfer path with PegaFlow's engine API.

Public surface (mirrors the reference's ``pegaflow.pegaflow`` module):
  PegaEngine, PyLoadState        in-process engine + shm load flag
  Executor, Layout, SaveSpec ... transfer executor (C ABI pf_executor_*)
"""

from ._native import PegaError, LIB_PATH  # noqa: F401  (loads the native library)
from .engine import PegaEngine, PyLoadState  # noqa: F401
from .transfer import (  # noqa: F401
    Executor,
    Layout,
    LoadSpec,
    PinnedBuffer,
    SaveSpec,
    refcopy_load,
    refcopy_save,
    segment_offset,
    validate,
)

__all__ = [
    "PegaEngine",
    "PyLoadState",
    "PegaError",
    "Executor",
    "Layout",
    "LoadSpec",
    "SaveSpec",
    "PinnedBuffer",
    "refcopy_save",
    "refcopy_load",
    "segment_offset",
    "validate",
]
