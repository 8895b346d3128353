"""CPU oracle for the KV block transfer path — TEST INFRASTRUCTURE ONLY.

Three independent restatements of the reference (xiaguan/pegaflow) algorithm:

  * ``liboracle`` (pf_oracle.c): per-layer save/load copies exactly as the
    reference worker issues them (gpu_worker.rs:205-372, transfer.rs:18-239);
  * numpy twins (``np_save_layer`` / ``np_load_layer``) of the same copies;
  * ``EngineModel``: the engine's host logic (lib.rs:373-1069, storage.rs)
    — registration checks, dedup, slot/seal, prefix hits, load selection —
    over host byte arrays;
  * ``dfs_pack`` / ``dfs_file_meta``: the packed-file tier's file bytes and
    metadata records (seal_offload.rs:79-105, 379-448).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module; the product library never does.

Parity status: KV-byte parity unpinned. The reference publishes no golden
vectors for KV bytes and its Rust sources cannot be built here (no Rust
toolchain), so parity of the byte path is defined by copy identity and pinned
against the reference's own tests
where they exist (LoadState header, allocator arithmetic) and against fixtures
generated from the reference's Python caller (tests/golden/). See the oracle
header in pf_oracle.c.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from collections import OrderedDict
from ctypes import POINTER, Structure, c_char_p, c_int, c_int64, c_size_t, c_uint8, c_uint64, c_void_p
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "pf_oracle.c"
OUT = HERE / "_build" / "liboracle.so"


def build(force: bool = False) -> Path:
    """Compile pf_oracle.c with gcc into oracle/_build/liboracle.so."""
    OUT.parent.mkdir(exist_ok=True)
    if force or not OUT.exists() or OUT.stat().st_mtime < SRC.stat().st_mtime:
        tmp = OUT.with_suffix(".so.tmp")
        subprocess.run(
            ["gcc", "-O2", "-std=c11", "-Wall", "-shared", "-fPIC", "-pthread", str(SRC), "-o", str(tmp)],
            check=True,
        )
        os.replace(tmp, OUT)
    return OUT


class OrLayout(Structure):
    _fields_ = [
        ("size_bytes", c_uint64),
        ("num_blocks", c_uint64),
        ("bytes_per_block", c_uint64),
        ("kv_stride_bytes", c_uint64),
        ("segments", c_uint64),
    ]


class OrMtLayer(Structure):
    _fields_ = [
        ("layout", OrLayout),
        ("gpu", c_void_p),
        ("ids", POINTER(c_int64)),
        ("n", c_uint64),
        ("k_pool", c_void_p),
        ("v_pool", c_void_p),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build()
        L = ctypes.CDLL(str(path))
        L.or_validate_layout.restype = c_int
        L.or_validate_layout.argtypes = [POINTER(OrLayout), c_char_p, c_char_p, c_size_t]
        L.or_segment_offset.restype = c_int
        L.or_segment_offset.argtypes = [POINTER(OrLayout), c_uint64, c_uint64, POINTER(c_uint64), c_char_p, c_size_t]
        L.or_save_layer.restype = c_int64
        L.or_save_layer.argtypes = [
            POINTER(OrLayout), c_void_p, POINTER(c_int64), c_uint64, c_void_p, c_void_p, c_char_p, c_size_t
        ]
        L.or_load_layer.restype = c_int64
        L.or_load_layer.argtypes = [
            POINTER(OrLayout), c_void_p, POINTER(c_int64), c_uint64, POINTER(c_void_p), POINTER(c_void_p), c_int,
            c_char_p, c_size_t,
        ]
        L.or_is_split.restype = c_int
        L.or_is_split.argtypes = [POINTER(OrLayout)]
        L.or_mt_transfer.restype = c_uint64
        L.or_mt_transfer.argtypes = [POINTER(OrMtLayer), c_uint64, c_int, c_int]
        _lib = L
    return _lib


@dataclass(frozen=True)
class Layout:
    size_bytes: int
    num_blocks: int
    bytes_per_block: int
    kv_stride_bytes: int
    segments: int

    def c(self) -> OrLayout:
        return OrLayout(self.size_bytes, self.num_blocks, self.bytes_per_block, self.kv_stride_bytes, self.segments)

    @property
    def split(self) -> bool:
        return self.segments == 2 and self.kv_stride_bytes > self.bytes_per_block

    @property
    def contiguous(self) -> bool:
        return self.segments <= 1 or self.kv_stride_bytes == self.bytes_per_block

    @property
    def block_size_bytes(self) -> int:
        return self.bytes_per_block * self.segments


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def validate_layout(layout: Layout, name: str = "") -> None:
    err = ctypes.create_string_buffer(512)
    rc = lib().or_validate_layout(ctypes.byref(layout.c()), name.encode(), err, 512)
    if rc:
        raise OracleError(rc, err.value.decode())


def segment_offset(layout: Layout, block: int, seg: int) -> int:
    err = ctypes.create_string_buffer(512)
    out = c_uint64()
    rc = lib().or_segment_offset(ctypes.byref(layout.c()), block, seg, ctypes.byref(out), err, 512)
    if rc:
        raise OracleError(rc, err.value.decode())
    return out.value


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def save_layer(layout: Layout, gpu: np.ndarray, ids: Sequence[int], k_dst: np.ndarray,
               v_dst: Optional[np.ndarray]) -> int:
    """process_save_task into k_dst/v_dst (uint8 arrays). Returns the reference's copy count."""
    ids_a = np.ascontiguousarray(ids, dtype=np.int64)
    err = ctypes.create_string_buffer(512)
    rc = lib().or_save_layer(
        ctypes.byref(layout.c()), _ptr(gpu), ids_a.ctypes.data_as(POINTER(c_int64)), ids_a.size, _ptr(k_dst),
        _ptr(v_dst) if v_dst is not None else None, err, 512,
    )
    if rc < 0:
        raise OracleError(-rc, err.value.decode())
    return rc


def load_layer(layout: Layout, gpu: np.ndarray, ids: Sequence[int], k_src: Sequence[int],
               v_src: Optional[Sequence[int]] = None, check_end: bool = True) -> int:
    """process_load_task for one layer; k_src/v_src are host addresses. Returns the run count."""
    ids_a = np.ascontiguousarray(ids, dtype=np.int64)
    ks = (c_void_p * max(1, len(k_src)))(*k_src)
    vs = (c_void_p * max(1, len(v_src)))(*v_src) if v_src is not None else None
    err = ctypes.create_string_buffer(512)
    rc = lib().or_load_layer(
        ctypes.byref(layout.c()), _ptr(gpu), ids_a.ctypes.data_as(POINTER(c_int64)), ids_a.size,
        ctypes.cast(ks, POINTER(c_void_p)), ctypes.cast(vs, POINTER(c_void_p)) if vs is not None else None,
        1 if check_end else 0, err, 512,
    )
    if rc < 0:
        raise OracleError(-rc, err.value.decode())
    return rc


# ----------------------------------------------------------------------------
# numpy twins (independent restatement of the same copies)
# ----------------------------------------------------------------------------

def np_save_layer(layout: Layout, gpu: np.ndarray, ids: Sequence[int]) -> tuple[np.ndarray, Optional[np.ndarray]]:
    """Pool bytes a save of `ids` produces: (K region, V region) for the split
    layout (lib.rs:639-679), else (block region, None) (lib.rs:707-747)."""
    ids = np.asarray(ids, dtype=np.int64)
    seg = layout.bytes_per_block
    if layout.split:
        k = np.stack([gpu[b * seg:(b + 1) * seg] for b in ids]) if len(ids) else np.zeros((0, seg), np.uint8)
        v = np.stack([gpu[layout.kv_stride_bytes + b * seg:layout.kv_stride_bytes + (b + 1) * seg] for b in ids]) \
            if len(ids) else np.zeros((0, seg), np.uint8)
        return k.reshape(-1), v.reshape(-1)
    bs = layout.block_size_bytes
    parts = []
    for b in ids:
        if layout.contiguous:
            parts.append(gpu[b * seg:b * seg + bs])
        else:
            parts.append(np.concatenate([gpu[b * seg + s * layout.kv_stride_bytes:b * seg + s * layout.kv_stride_bytes + seg]
                                         for s in range(layout.segments)]))
    return (np.concatenate(parts) if parts else np.zeros(0, np.uint8)), None


def np_load_layer(layout: Layout, gpu: np.ndarray, ids: Sequence[int], k_bytes: Sequence[np.ndarray],
                  v_bytes: Optional[Sequence[np.ndarray]]) -> None:
    """Write block payloads back into `gpu` in list order (later ids win), as
    process_load_task's copies do (gpu_worker.rs:223-282)."""
    seg = layout.bytes_per_block
    for i, b in enumerate(ids):
        if layout.split:
            gpu[b * seg:(b + 1) * seg] = k_bytes[i][:seg]
        else:
            gpu[b * seg:b * seg + layout.block_size_bytes] = k_bytes[i][:layout.block_size_bytes]
    if layout.split:
        for i, b in enumerate(ids):
            o = layout.kv_stride_bytes + b * seg
            gpu[o:o + seg] = v_bytes[i][:seg] if v_bytes is not None else k_bytes[i][seg:2 * seg]


# ----------------------------------------------------------------------------
# Engine model (lib.rs:93-1069 + storage.rs, LRU without TinyLFU admission)
# ----------------------------------------------------------------------------

@dataclass
class _Slot:
    k: np.ndarray                  # K (or whole block) payload bytes
    v: Optional[np.ndarray]        # V payload bytes (split)


@dataclass
class _Instance:
    ns: str
    num_layers: int
    tp_size: int
    layer_ids: dict = field(default_factory=dict)
    regs: dict = field(default_factory=dict)  # (device, layer) -> (Layout, gpu array)


class EngineModel:
    """Host-logic restatement of PegaEngine with byte payloads.

    The pool is unbounded (no eviction); payloads are copied out of the
    layer's "GPU" array at save time and written back on load.
    """

    def __init__(self):
        self.instances: dict[str, _Instance] = {}
        self.inflight: dict[tuple[str, bytes], list] = {}
        self.cache: "OrderedDict[tuple[str, bytes], list]" = OrderedDict()

    def register_context_layer(self, instance_id, namespace, device_id, layer_name, gpu: np.ndarray,
                               layout: Layout, tp_rank, tp_size, num_layers):
        validate_layout(layout, layer_name)
        if device_id < 0:
            raise OracleError(3, "invalid argument: device_id must be >= 0")
        inst = self.instances.get(instance_id)
        if inst is not None and (inst.num_layers != num_layers or inst.tp_size != tp_size):
            raise OracleError(7, f"topology mismatch: instance {instance_id} exists with layers={inst.num_layers}, "
                                 f"tp={inst.tp_size}; requested layers={num_layers}, tp={tp_size}")
        if inst is None:
            inst = self.instances[instance_id] = _Instance(namespace, num_layers, tp_size)
        inst.layer_ids.setdefault(layer_name, len(inst.layer_ids))
        inst.regs[(device_id, layer_name)] = (layout, gpu)

    def unregister_instance(self, instance_id):
        if self.instances.pop(instance_id, None) is None:
            raise OracleError(1, f"instance {instance_id} not found")

    def _inst(self, instance_id) -> _Instance:
        if instance_id not in self.instances:
            raise OracleError(1, f"instance {instance_id} not found")
        return self.instances[instance_id]

    def _slot(self, inst, layer_id, tp_rank):
        if layer_id >= inst.num_layers:
            raise OracleError(3, f"invalid argument: layer_id {layer_id} out of range ({inst.num_layers} layers)")
        if tp_rank >= inst.tp_size:
            raise OracleError(3, f"invalid argument: tp_rank {tp_rank} out of range (tp_size {inst.tp_size})")
        return layer_id * inst.tp_size + tp_rank

    def batch_save(self, instance_id, tp_rank, device_id, saves):
        """batch_save_kv_blocks_from_ipc: entries one after another (lib.rs:507-518)."""
        inst = self._inst(instance_id)
        for layer_name, ids, hashes in saves:
            self._save_inner(inst, instance_id, tp_rank, device_id, layer_name, list(ids), [bytes(h) for h in hashes])

    def _save_inner(self, inst, instance_id, tp_rank, device_id, layer_name, ids, hashes):
        if len(ids) != len(hashes):
            raise OracleError(3, f"invalid argument: block_ids length {len(ids)} does not match block_hashes {len(hashes)}")
        if not any(d == device_id for d, _ in inst.regs):
            raise OracleError(2, f"device {device_id} not found in instance {instance_id}")
        if layer_name not in inst.layer_ids:
            raise OracleError(3, f"invalid argument: layer {layer_name} unknown")
        if (device_id, layer_name) not in inst.regs:
            raise OracleError(3, f"invalid argument: layer {layer_name} not registered on device")
        layout, gpu = inst.regs[(device_id, layer_name)]
        slot = self._slot(inst, inst.layer_ids[layer_name], tp_rank)
        total = inst.num_layers * inst.tp_size
        todo = []
        for b, h in zip(ids, hashes):
            if b < 0:
                continue
            if b >= layout.num_blocks:
                raise OracleError(3, f"invalid argument: block {b} out of range for layer {layer_name} "
                                     f"({layout.num_blocks} blocks registered)")
            key = (inst.ns, h)
            in_flight = key in self.inflight and self.inflight[key][slot] is not None
            if key not in self.cache and not in_flight:
                todo.append((b, h))
        if not todo:
            return
        # The pool bytes of this save, via the C restatement of the worker copies.
        n = len(todo)
        seg = layout.bytes_per_block
        if layout.split:
            kreg = np.zeros(n * seg, np.uint8)
            vreg = np.zeros(n * seg, np.uint8)
            save_layer(layout, gpu, [b for b, _ in todo], kreg, vreg)
            payloads = [_Slot(kreg[i * seg:(i + 1) * seg].copy(), vreg[i * seg:(i + 1) * seg].copy()) for i in range(n)]
        else:
            bs = layout.block_size_bytes
            reg = np.zeros(n * bs, np.uint8)
            save_layer(layout, gpu, [b for b, _ in todo], reg, None)
            payloads = [_Slot(reg[i * bs:(i + 1) * bs].copy(), None) for i in range(n)]
        for (b, h), p in zip(todo, payloads):
            self._insert_slot(inst.ns, h, slot, p, total)

    def _insert_slot(self, ns, h, slot, payload, total):
        key = (ns, h)
        if key in self.cache:
            return False
        blk = self.inflight.setdefault(key, [None] * total)
        if blk[slot] is not None:
            return False
        blk[slot] = payload
        if all(s is not None for s in blk):
            del self.inflight[key]
            self.cache[key] = blk
        return True

    def count_prefix_hit_blocks(self, instance_id, hashes):
        inst = self._inst(instance_id)
        hit = 0
        for h in hashes:
            if (inst.ns, bytes(h)) not in self.cache:
                break
            hit += 1
        return hit

    def batch_load(self, instance_id, tp_rank, device_id, layer_names, ids, hashes):
        """batch_load_kv_blocks_multi_layer + process_load_task; returns the
        LoadState value the reference ends with (1 or -1) and the error, if any."""
        try:
            inst = self._inst(instance_id)
            if not any(d == device_id for d, _ in inst.regs):
                raise OracleError(2, f"device {device_id} not found in instance {instance_id}")
            blocks = []
            for i, h in enumerate(hashes):
                key = (inst.ns, bytes(h))
                if key not in self.cache:
                    raise OracleError(5, f"storage error: missing KV block hash at index {i} "
                                         f"(namespace={inst.ns}, hash_len={len(h)})")
                self.cache.move_to_end(key)
                blocks.append(self.cache[key])
            work = []
            for name in layer_names:
                if name not in inst.layer_ids:
                    raise OracleError(3, f"invalid argument: layer {name} unknown for instance {instance_id}")
                if (device_id, name) not in inst.regs:
                    raise OracleError(3, f"invalid argument: layer {name} not registered on device {device_id}")
                slot = self._slot(inst, inst.layer_ids[name], tp_rank)
                sel = [(b, blk[slot]) for b, blk in zip(ids, blocks) if b >= 0]
                if sel:
                    work.append((name, sel))
        except OracleError as e:
            return -1, e
        # Worker: check every offset first, then copy (the B200 library validates
        # the whole task before moving bytes).
        try:
            for name, sel in work:
                layout, gpu = inst.regs[(device_id, name)]
                for b, _ in sel:
                    segment_offset(layout, b, 0)
                    if layout.split:
                        segment_offset(layout, b, 1)
                    elif b * layout.bytes_per_block + layout.block_size_bytes > layout.size_bytes:
                        raise OracleError(5, f"Block {b} exceeds registered memory")
        except OracleError as e:
            return -1, e
        for name, sel in work:
            layout, gpu = inst.regs[(device_id, name)]
            np_load_layer(layout, gpu, [b for b, _ in sel], [p.k for _, p in sel],
                          [p.v for _, p in sel] if layout.split else None)
        return 1, None

    def slot_payload(self, ns, h, slot):
        blk = self.cache.get((ns, bytes(h)))
        return None if blk is None else blk[slot]


# ----------------------------------------------------------------------------
# CPU baseline
# ----------------------------------------------------------------------------

def mt_transfer(layers: Sequence[tuple[Layout, np.ndarray, np.ndarray, np.ndarray, Optional[np.ndarray]]],
                save: bool, threads: int) -> int:
    """Multi-threaded gather (save) / scatter (load) of split or contiguous
    layers between host "KV cache" arrays and pool arrays. Each layer is
    (layout, gpu_bytes, ids, k_pool, v_pool). Returns payload bytes moved."""
    arr = (OrMtLayer * max(1, len(layers)))()
    keep = []
    for i, (layout, gpu, ids, kp, vp) in enumerate(layers):
        ids_a = np.ascontiguousarray(ids, dtype=np.int64)
        keep.append(ids_a)
        arr[i].layout = layout.c()
        arr[i].gpu = _ptr(gpu)
        arr[i].ids = ids_a.ctypes.data_as(POINTER(c_int64))
        arr[i].n = ids_a.size
        arr[i].k_pool = _ptr(kp)
        arr[i].v_pool = _ptr(vp) if vp is not None else None
    return lib().or_mt_transfer(arr, len(layers), 1 if save else 0, threads)


# ----------------------------------------------------------------------------
# Packed-file tier (seal_offload.rs)
# ----------------------------------------------------------------------------

def dfs_pack(blocks, file_name: str):
    """write_packed_file (seal_offload.rs:379-448) restated. ``blocks`` is a
    list of sealed blocks, each a list of slots ``(k_bytes, v_bytes or None)``
    with a slot's size = len(k) + len(v). Returns the packed file's bytes and
    each block's BlockMeta record as serde_json writes it (compact, fields in
    declaration order: file, offset, slots[is_split, size], total_slots)."""
    import json

    total_slots = len(blocks[0]) if blocks else 0
    data, metas, offset = bytearray(), [], 0
    for slots in blocks:
        slot_meta = []
        for k, v in slots:
            data += bytes(k)
            if v is not None:
                data += bytes(v)
            slot_meta.append({"is_split": v is not None, "size": len(k) + (len(v) if v is not None else 0)})
        metas.append(json.dumps({"file": file_name, "offset": offset, "slots": slot_meta,
                                 "total_slots": total_slots}, separators=(",", ":")))
        offset += sum(s["size"] for s in slot_meta)
    return bytes(data), metas


def dfs_file_meta(hashes, size: int) -> str:
    """FileMeta (seal_offload.rs:100-105) as serde_json writes it."""
    import json

    return json.dumps({"blocks": [bytes(h).hex() for h in hashes], "size": size}, separators=(",", ":"))
