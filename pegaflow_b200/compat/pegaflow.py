"""Stand-in for the reference's compiled extension module ``pegaflow.pegaflow``.

The reference's Python package (``pegaflow``: the vLLM connector, the SGLang
adapter, the CUDA IPC wrapper) takes its engine classes from the PyO3
extension ``pegaflow.pegaflow`` (python/src/lib.rs:579-585), imported by
python/pegaflow/__init__.py:10, connector/common.py:14 and connector/worker.py:18.
This file, placed in that package as ``pegaflow/pegaflow.py`` in place of the
compiled extension (``python -m pegaflow_b200.compat <package dir>`` does it),
makes the package's unmodified code run on this library: its connector's
``EngineRpcClient`` talks to ``python -m pegaflow_b200.server`` over the same
gRPC surface, and in-process callers get this library's ``PegaEngine`` and
``PyLoadState``.
"""

from pegaflow_b200.client import EngineRpcClient
from pegaflow_b200.engine import PegaEngine, PyLoadState

__all__ = ["EngineRpcClient", "PegaEngine", "PyLoadState"]
