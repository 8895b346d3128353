"""Python view of the transfer executor (pf_executor_* in include/pegaflow.h).

The executor is the B200 replacement for the reference's per-device worker
copy loops (pegaflow-core/src/gpu_worker.rs:205-390): a save gathers the
listed blocks of each layer into the pinned pool with an sm_100a pack kernel
plus copy-engine DMA, a load scatters pool bytes back into arbitrary block ids.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, byref, c_int64, c_uint64, c_void_p
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _native as N

_MODES = {"auto": N.PF_MODE_AUTO, "staged": N.PF_MODE_STAGED, "direct": N.PF_MODE_DIRECT}
_COPY_KERNELS = {"auto": N.PF_COPY_KERNEL_AUTO, "registers": N.PF_COPY_KERNEL_REGISTERS,
                 "bulk": N.PF_COPY_KERNEL_BULK}


@dataclass(frozen=True)
class Layout:
    """KVCacheRegistration (pegaflow-core/src/lib.rs:100-112)."""

    data_ptr: int
    size_bytes: int
    num_blocks: int
    bytes_per_block: int
    kv_stride_bytes: int
    segments: int

    @staticmethod
    def from_tensor(t) -> "Layout":
        """Layout of a paged KV tensor, derived as the vLLM connector does
        (python/pegaflow/connector/worker.py:100-115): a leading dimension of 2
        is KV-first (segments=2), anything else is blocks-first."""
        shape, stride, elt = tuple(t.shape), tuple(t.stride()), t.element_size()
        if len(shape) >= 2 and shape[0] == 2:
            return Layout(t.data_ptr(), t.numel() * elt, shape[1], stride[1] * elt, stride[0] * elt, 2)
        return Layout(t.data_ptr(), t.numel() * elt, shape[0], stride[0] * elt, 0, 1)

    @staticmethod
    def from_token_major(t, page_size: int) -> "Layout":
        """Layout of a token-major K or V buffer ``[slots, heads, head_dim]``
        whose pages of ``page_size`` tokens are the blocks, registered as one
        segments=1 layer, as the SGLang adapter derives it
        (python/pegaflow/sglang/peagflow_radix_cache.py:203-222)."""
        if page_size <= 0:
            raise ValueError("page_size must be > 0")
        slots, elt = t.shape[0], t.element_size()
        if slots % page_size:
            raise ValueError(f"KV slots ({slots}) must be divisible by page_size ({page_size})")
        return Layout(t.data_ptr(), t.numel() * elt, slots // page_size, t.stride(0) * elt * page_size, 0, 1)

    def c(self) -> N.LayerDesc:
        return N.LayerDesc(
            self.data_ptr, self.size_bytes, self.num_blocks, self.bytes_per_block, self.kv_stride_bytes, self.segments
        )

    @property
    def split(self) -> bool:
        return self.segments == 2 and self.kv_stride_bytes > self.bytes_per_block

    @property
    def block_size_bytes(self) -> int:
        return self.bytes_per_block * self.segments


def validate(layout: Layout, name: str = "") -> None:
    N.check(N.lib.pf_layer_validate(byref(layout.c()), name.encode()))


def segment_offset(layout: Layout, block_idx: int, segment_idx: int) -> int:
    out = c_uint64()
    N.check(N.lib.pf_segment_offset(byref(layout.c()), block_idx, segment_idx, byref(out)))
    return out.value


@dataclass
class SaveSpec:
    """One layer of a save: block i of ``block_idx`` lands at ``k_dst + i*pitch``
    (and ``v_dst + i*bytes_per_block`` for the split K/V layout)."""

    layout: Layout
    block_idx: np.ndarray
    k_dst: int
    v_dst: Optional[int] = None


@dataclass
class LoadSpec:
    """One layer of a load: host K/V pointers per block (LayerBlock k_ptr/v_ptr)."""

    layout: Layout
    block_idx: np.ndarray
    k_src: np.ndarray
    v_src: Optional[np.ndarray] = None


@dataclass
class P2PSpec:
    """One layer of a GPU-to-GPU handoff: block src_idx[i] of `src` lands in
    block dst_idx[i] of `dst` (same bytes_per_block, segments and K/V split)."""

    src: Layout
    dst: Layout
    src_idx: np.ndarray
    dst_idx: np.ndarray


def _p2p_array(specs: Sequence[P2PSpec]):
    arr = (N.P2PLayer * max(1, len(specs)))()
    keep = []
    for i, s in enumerate(specs):
        a = np.ascontiguousarray(s.src_idx, dtype=np.int64)
        b = np.ascontiguousarray(s.dst_idx, dtype=np.int64)
        if a.size != b.size:
            raise ValueError("src_idx and dst_idx differ in length")
        keep += [a, b]
        arr[i].src = s.src.c()
        arr[i].dst = s.dst.c()
        arr[i].src_idx = a.ctypes.data_as(POINTER(c_int64))
        arr[i].dst_idx = b.ctypes.data_as(POINTER(c_int64))
        arr[i].n = a.size
    return arr, keep


def _save_array(specs: Sequence[SaveSpec]):
    arr = (N.SaveLayer * max(1, len(specs)))()
    keep = []
    for i, s in enumerate(specs):
        ids = np.ascontiguousarray(s.block_idx, dtype=np.int64)
        keep.append(ids)
        arr[i].layer = s.layout.c()
        arr[i].block_idx = ids.ctypes.data_as(POINTER(c_int64))
        arr[i].n = ids.size
        arr[i].k_dst = s.k_dst
        arr[i].v_dst = s.v_dst or None
    return arr, keep


def _load_array(specs: Sequence[LoadSpec]):
    arr = (N.LoadLayer * max(1, len(specs)))()
    keep = []
    for i, s in enumerate(specs):
        ids = np.ascontiguousarray(s.block_idx, dtype=np.int64)
        ks = np.ascontiguousarray(s.k_src, dtype=np.uint64)
        keep += [ids, ks]
        arr[i].layer = s.layout.c()
        arr[i].block_idx = ids.ctypes.data_as(POINTER(c_int64))
        arr[i].n = ids.size
        arr[i].k_src = ks.ctypes.data_as(POINTER(c_void_p))
        if s.v_src is not None:
            vs = np.ascontiguousarray(s.v_src, dtype=np.uint64)
            keep.append(vs)
            arr[i].v_src = vs.ctypes.data_as(POINTER(c_void_p))
        else:
            arr[i].v_src = None
    return arr, keep


class Executor:
    """Per-device transfer executor (pf_executor)."""

    def __init__(
        self,
        device_id: int = 0,
        *,
        staging_chunk_bytes: int = 0,
        staging_slots: int = 0,
        save_mode: str = "auto",
        load_mode: str = "auto",
        ctas_per_sm: int = 0,
        copy_streams: int = 0,
        cache_streaming: bool = False,
        first_chunk_bytes: int = 0,
        copy_kernel: str = "auto",
        _handle: Optional[int] = None,
    ):
        self.device_id = device_id
        self._owned = _handle is None
        if _handle is not None:
            self._h = c_void_p(_handle)
            return
        cfg = N.ExecutorConfig()
        N.lib.pf_executor_config_default(byref(cfg))
        if staging_chunk_bytes:
            cfg.staging_chunk_bytes = staging_chunk_bytes
        if staging_slots:
            cfg.staging_slots = staging_slots
        cfg.save_mode = _MODES[save_mode]
        cfg.load_mode = _MODES[load_mode]
        if ctas_per_sm:
            cfg.ctas_per_sm = ctas_per_sm
        if copy_streams:
            cfg.copy_streams = copy_streams
        cfg.cache_streaming = 1 if cache_streaming else 0
        if first_chunk_bytes:
            cfg.first_chunk_bytes = first_chunk_bytes
        cfg.copy_kernel = _COPY_KERNELS[copy_kernel]
        h = c_void_p()
        N.check(N.lib.pf_executor_create(device_id, byref(cfg), byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None) and self._owned:
            N.lib.pf_executor_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def save(self, specs: Sequence[SaveSpec], stream: Optional[int] = None) -> None:
        """Blocking save, or stream-ordered when ``stream`` (a cudaStream_t as int) is given."""
        arr, keep = _save_array(specs)
        if stream is None:
            N.check(N.lib.pf_save_blocks(self._h, arr, len(specs)))
        else:
            N.check(N.lib.pf_save_blocks_async(self._h, arr, len(specs), c_void_p(stream)))
        del keep

    def load(self, specs: Sequence[LoadSpec], stream: Optional[int] = None, layer_done: Optional[int] = None) -> None:
        arr, keep = _load_array(specs)
        if stream is None and layer_done is None:
            N.check(N.lib.pf_load_blocks(self._h, arr, len(specs)))
        else:
            N.check(
                N.lib.pf_load_blocks_async(
                    self._h, arr, len(specs), c_void_p(stream or 0), c_void_p(layer_done) if layer_done else None
                )
            )
        del keep

    def p2p(self, specs: Sequence[P2PSpec], peer_device: int, push: bool = False,
            stream: Optional[int] = None) -> None:
        """GPU-to-GPU paged copy over NVLink. pull (default): this executor's
        device holds the destinations and reads the peer's blocks; push: this
        device holds the sources and writes into the peer's blocks."""
        arr, keep = _p2p_array(specs)
        N.check(N.lib.pf_p2p_transfer(self._h, peer_device, 1 if push else 0, arr, len(specs),
                                      c_void_p(stream) if stream else None))
        del keep

    def stats(self) -> dict:
        s = N.ExecutorStats()
        N.check(N.lib.pf_executor_stats_get(self._h, byref(s)))
        return {f: getattr(s, f) for f, _ in N.ExecutorStats._fields_}

    def reset_stats(self) -> None:
        N.check(N.lib.pf_executor_stats_reset(self._h))

    def set_timing(self, on: bool) -> None:
        N.check(N.lib.pf_executor_set_timing(self._h, 1 if on else 0))


def refcopy_save(device_id: int, specs: Sequence[SaveSpec]) -> None:
    """The reference's save copy strategy (one synchronous D2H per segment)."""
    arr, keep = _save_array(specs)
    N.check(N.lib.pf_refcopy_save(device_id, arr, len(specs)))
    del keep


def refcopy_load(device_id: int, specs: Sequence[LoadSpec]) -> int:
    """The reference's load copy strategy (merged runs, one H2D each); returns the run count."""
    arr, keep = _load_array(specs)
    runs = c_uint64()
    N.check(N.lib.pf_refcopy_load(device_id, arr, len(specs), byref(runs)))
    del keep
    return runs.value


class PinnedBuffer:
    """Pinned, mapped host memory from pf_pinned_alloc, viewable as numpy."""

    def __init__(self, nbytes: int, write_combined: bool = False):
        p = c_void_p()
        N.check(N.lib.pf_pinned_alloc(nbytes, 1 if write_combined else 0, byref(p)))
        self.ptr = p.value
        self.nbytes = nbytes

    def numpy(self, dtype=np.uint8) -> np.ndarray:
        buf = (ctypes.c_uint8 * self.nbytes).from_address(self.ptr)
        return np.frombuffer(buf, dtype=np.uint8).view(dtype)

    def close(self) -> None:
        if self.ptr:
            N.check(N.lib.pf_pinned_free(c_void_p(self.ptr)))
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
