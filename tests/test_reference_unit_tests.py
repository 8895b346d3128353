"""The reference's own unit tests, restated against this library (CPU only).

pegaflow-core/src/sync_state.rs:294-341   (LoadState)
pegaflow-core/src/allocator.rs:179-239    (ScaledOffsetAllocator)
pegaflow-core/src/pinned_mem.rs:284-288   (zero-size pinned allocation)
These are the only known-answer tests the reference holds for this path.
"""

import mmap
import os
import uuid
from ctypes import byref, c_uint32, c_uint64, c_void_p
from pathlib import Path

import _posixshmem
import pytest

U32_MAX = 2**32 - 1


# --------------------------------------------------------------------------- LoadState


def test_load_state_create_and_attach_round_trip(native):
    from pegaflow_b200 import PyLoadState

    s = PyLoadState()
    assert s.get_state() == 0
    name = s.shm_name()
    s.set_completed()
    a = PyLoadState.attach(name)
    assert a.get_state() == 1
    a.close()
    s.close()


def test_load_state_attach_rejects_too_small_mapping(native):
    from pegaflow_b200 import PyLoadState

    name = f"pega_test_small_{uuid.uuid4().hex}"
    fd = _posixshmem.shm_open(name, os.O_CREAT | os.O_EXCL | os.O_RDWR, mode=0o600)
    try:
        os.ftruncate(fd, 1)
        with pytest.raises(RuntimeError, match="shared memory too small") as ei:
            PyLoadState.attach(name)
        assert ei.value.code == native.PF_ERR_LOAD_STATE
    finally:
        os.close(fd)
        _posixshmem.shm_unlink(name)


def test_load_state_attach_rejects_invalid_header(native):
    from pegaflow_b200 import PyLoadState

    s = PyLoadState()
    path = Path("/dev/shm") / s.shm_name()
    with open(path, "r+b") as f:
        m = mmap.mmap(f.fileno(), 32)
        offset = int.from_bytes(m[0:8], "little")
        m[offset:offset + 4] = (0xDEADBEEF).to_bytes(4, "little")
        m.close()
    with pytest.raises(RuntimeError, match="invalid LoadState header"):
        PyLoadState.attach(s.shm_name())
    s.close()


def test_load_state_byte_layout_matches_reference(native):
    """[usize offset=8][u32 magic 'PFLD'][u32 version 1][i64 state], 32 bytes
    (sync_state.rs:27-43,186-193); name pega_load_<32 hex> (sync_state.rs:126)."""
    from pegaflow_b200 import PyLoadState

    s = PyLoadState()
    name = s.shm_name()
    assert name.startswith("pega_load_") and len(name) == len("pega_load_") + 32
    int(name[len("pega_load_"):], 16)
    raw = (Path("/dev/shm") / name).read_bytes()
    assert len(raw) == 32
    assert raw[0:8] == (8).to_bytes(8, "little")
    assert raw[8:12] == (0x50464C44).to_bytes(4, "little")
    assert raw[12:16] == (1).to_bytes(4, "little")
    assert raw[16:24] == (0).to_bytes(8, "little", signed=True)
    s.set_error()
    raw = (Path("/dev/shm") / name).read_bytes()
    assert int.from_bytes(raw[16:24], "little", signed=True) == -1
    s.close()
    assert not (Path("/dev/shm") / name).exists(), "the creating handle unlinks on close"


def test_load_state_layer_extension_keeps_version_1_bytes(native):
    """The per-layer extension sits after the 32 version-1 bytes; a reader that
    validates only those (sync_state.rs:244-292) attaches unchanged."""
    from pegaflow_b200 import PyLoadState

    s = PyLoadState(5)
    raw = (Path("/dev/shm") / s.shm_name()).read_bytes()
    assert len(raw) == 32 + 16 + 5 * 8
    assert raw[0:8] == (8).to_bytes(8, "little") and raw[8:12] == (0x50464C44).to_bytes(4, "little")
    assert raw[12:16] == (1).to_bytes(4, "little")
    assert raw[32:36] == b"PFL2" and int.from_bytes(raw[36:40], "little") == 5
    a = PyLoadState.attach(s.shm_name())
    assert a.layer_count() == 5 and not any(a.layer_ready(i) for i in range(5))
    assert PyLoadState().layer_count() == 0
    a.close()
    s.close()


# --------------------------------------------------------------------------- allocator


class Alloc:
    def __init__(self, native, total, unit, max_allocs=0):
        self.n = native
        h = c_void_p()
        native.check(native.lib.pf_allocator_create(total, unit, max_allocs, byref(h)))
        self.h = h

    def alloc(self, size):
        off, sz, hd = c_uint64(), c_uint64(), c_uint32()
        rc = self.n.lib.pf_allocator_alloc(self.h, size, byref(off), byref(sz), byref(hd))
        if rc == self.n.PF_ERR_NO_SPACE:
            return None
        self.n.check(rc)
        return off.value, sz.value, hd.value

    def free(self, a):
        self.n.lib.pf_allocator_free(self.h, a[2])

    def report(self):
        tf, lf, tb, us = c_uint64(), c_uint64(), c_uint64(), c_uint64()
        self.n.lib.pf_allocator_report(self.h, byref(tf), byref(lf), byref(tb), byref(us))
        return tf.value, lf.value, tb.value, us.value

    def __del__(self):
        self.n.lib.pf_allocator_destroy(self.h)


def test_allocator_creates_with_scaled_capacity(native):
    a = Alloc(native, 10 * 1024**3, 64)
    _, _, total, unit = a.report()
    assert unit == 64
    assert total // unit == (10 * 1024**3) // 64


def test_allocator_allocate_rounds_up_to_unit_size(native):
    a = Alloc(native, 1024, 64)
    off, size, _ = a.alloc(1)
    assert (off, size) == (0, 64)
    total_free, largest, _, _ = a.report()
    assert (total_free, largest) == (960, 960)


def test_allocator_reuse_after_free_merges_neighboring_regions(native):
    a = Alloc(native, 256, 64)
    x = a.alloc(64)
    y = a.alloc(64)
    a.free(x)
    a.free(y)
    merged = a.alloc(128)
    assert merged[:2] == (0, 128)


def test_allocator_rejects_unreasonably_large_requests(native):
    a = Alloc(native, 1024 * 1024, 1)
    h = a.h
    off, sz, hd = c_uint64(), c_uint64(), c_uint32()
    rc = native.lib.pf_allocator_alloc(h, U32_MAX * 2, byref(off), byref(sz), byref(hd))
    assert rc == native.PF_ERR_INVALID_ARGUMENT
    assert "overflows u32" in native.lib.pf_last_error().decode()


def test_allocator_rejects_invalid_unit_size(native):
    h = c_void_p()
    rc = native.lib.pf_allocator_create(1024, 0, 0, byref(h))
    assert rc == native.PF_ERR_INVALID_ARGUMENT
    assert "unit size must be greater than zero" in native.lib.pf_last_error().decode()


def test_allocator_auto_unit_follows_code(native):
    """ScaledOffsetAllocator::new picks ceil(total / u32::MAX) (allocator.rs:77-86):
    17-byte units for 64 GiB (the comment there says 16; the code decides)."""
    a = Alloc(native, 64 * 1024**3, native.PF_ALLOCATOR_AUTO_UNIT)
    assert a.report()[3] == -(-64 * 1024**3 // U32_MAX) == 17
    b = Alloc(native, 1 << 20, native.PF_ALLOCATOR_AUTO_UNIT)
    assert b.report()[3] == 1


def test_allocator_exhaustion_and_reclaim_sequence(native):
    """No space -> None (allocator.rs:138-140); freeing makes room again."""
    a = Alloc(native, 64 * 10, 64)
    held = [a.alloc(64) for _ in range(10)]
    assert all(h is not None for h in held)
    assert a.alloc(64) is None
    a.free(held[3])
    assert a.alloc(64)[0] == 3 * 64


# --------------------------------------------------------------------------- pinned memory


def test_pinned_zero_size_fails(native):
    p = c_void_p()
    rc = native.lib.pf_pinned_alloc(0, 1, byref(p))
    assert rc == native.PF_ERR_INVALID_ARGUMENT
    assert "size must be greater than zero" in native.lib.pf_last_error().decode()
