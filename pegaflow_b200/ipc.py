"""CUDA IPC wrapper for handing KV tensors to the engine server process.

The vLLM worker pickles a wrapper of each KV tensor into RegisterContext's
``wrapper_bytes`` (python/pegaflow/connector/worker.py:97-98); the server
unpickles it and maps the memory (pegaflow-server/src/registry.rs:144-175).
The pickled state — attributes ``handle`` (torch's CUDA storage share
tuple), ``dtype``, ``shape`` and ``device_uuid`` — is the interface between
the two processes and is kept as the reference defines it
(python/pegaflow/ipc_wrapper.py:101-122), so bytes produced by either side's
wrapper load here.

Unpickling runs with a restricted loader: only the wrapper class (under this
module or the reference's ``pegaflow.ipc_wrapper`` path), ``torch.Size`` and
torch dtypes may be named, so wrapper bytes cannot execute arbitrary code.
"""

from __future__ import annotations

import io
import pickle
import threading


class CudaIPCWrapper:
    """A CUDA tensor's IPC handle plus what is needed to rebuild the tensor
    in another process. Devices are identified by UUID so the receiver maps
    the right GPU whatever its CUDA_VISIBLE_DEVICES."""

    _uuid_to_index: dict = {}
    _lock = threading.Lock()

    def __init__(self, tensor):
        if tensor.storage_offset() != 0:
            raise ValueError("KV tensor must start at its storage's first byte")
        if not tensor.is_contiguous():
            raise ValueError("KV tensor must be contiguous")
        import torch

        self.handle = tensor.untyped_storage()._share_cuda_()
        self.dtype = tensor.dtype
        self.shape = tensor.shape
        self.device_uuid = str(torch.cuda.get_device_properties(tensor.device.index).uuid)

    @classmethod
    def _device_of(cls, uuid: str) -> int:
        import torch

        with cls._lock:
            if not cls._uuid_to_index:
                for i in range(torch.cuda.device_count()):
                    cls._uuid_to_index[str(torch.cuda.get_device_properties(i).uuid)] = i
            index = cls._uuid_to_index.get(uuid)
        if index is None:
            raise RuntimeError(f"GPU {uuid} is not visible to this process")
        return index

    def to_tensor(self):
        """Map the shared memory in this process (the storage stays alive as
        long as the returned tensor does)."""
        import torch

        device = self._device_of(self.device_uuid)
        storage = torch.UntypedStorage._new_shared_cuda(device, *self.handle[1:])
        t = torch.empty(0, device=device, dtype=self.dtype)
        t.set_(storage)
        return t.view(self.shape)

    def __repr__(self) -> str:
        return f"CudaIPCWrapper(shape={tuple(self.shape)}, dtype={self.dtype}, device_uuid={self.device_uuid})"


_WRAPPER_PATHS = {("pegaflow.ipc_wrapper", "CudaIPCWrapper"), (__name__, "CudaIPCWrapper")}


class _WrapperUnpickler(pickle.Unpickler):
    def find_class(self, module, name):
        if (module, name) in _WRAPPER_PATHS:
            return CudaIPCWrapper
        if module == "torch":
            import torch

            obj = getattr(torch, name, None)
            if name == "Size" or isinstance(obj, torch.dtype):
                return obj
        raise pickle.UnpicklingError(f"wrapper bytes may not reference {module}.{name}")


def loads_wrapper(data: bytes) -> CudaIPCWrapper:
    """Unpickle RegisterContext.wrapper_bytes with the restricted loader."""
    obj = _WrapperUnpickler(io.BytesIO(data)).load()
    if not isinstance(obj, CudaIPCWrapper):
        raise pickle.UnpicklingError(f"wrapper bytes hold a {type(obj).__name__}, not a CudaIPCWrapper")
    return obj
