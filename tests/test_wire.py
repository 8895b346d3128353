"""The native decoder of the gRPC server's Save and Load requests
(pegaflow_b200/csrc/wire.cpp, through tests/wire_test.cpp) against the
protobuf library's parse of the same wire bytes (engine.proto, field numbers
as in pegaflow-proto/proto/engine.proto:5-115):

- random requests serialised by the protobuf library (negative ids and
  device ids, empty and odd-length hashes, many layers, layers sharing one
  hash list);
- hand-written wire bytes the library would also accept: unpacked block ids,
  fields out of order, unknown fields of every wire type, a singular field
  given twice (the last one wins);
- truncated and malformed bytes, which must fail cleanly;
- layers whose hash lists are equal share one list, and only those.
"""

import os
import random
import subprocess
from pathlib import Path

import pytest

from pegaflow_b200 import proto as P

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "pegaflow_b200" / "csrc"
CUDA = Path("/usr/local/cuda")


@pytest.fixture(scope="module")
def wire_test():
    exe = ROOT / "tests" / "_build" / "wire_test"
    exe.parent.mkdir(exist_ok=True)
    cmd = ["g++", "-O1", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA / 'include'}",
           str(ROOT / "tests" / "wire_test.cpp"), str(CSRC / "wire.cpp"), "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def run(exe, mode, data: bytes, tmp_path):
    f = tmp_path / "req.bin"
    f.write_bytes(data)
    p = subprocess.run([str(exe), mode, str(f)], capture_output=True, text=True, timeout=60)
    return p.returncode, p.stdout


def want_save(req) -> str:
    lines = [f"instance_id={req.instance_id.encode().hex()}", f"tp_rank={req.tp_rank}",
             f"device_id={req.device_id}", f"layers={len(req.saves)}"]
    prev = None
    for i, s in enumerate(req.saves):
        hashes = list(s.block_hashes)
        shared = int(i > 0 and hashes == prev)
        lines.append(f"layer {i} name={s.layer_name.encode().hex()} ids={','.join(map(str, s.block_ids))} "
                     f"hashes={','.join(h.hex() for h in hashes)} shared={shared}")
        prev = hashes
    return "\n".join(lines) + "\n"


def want_load(req) -> str:
    return "\n".join([f"instance_id={req.instance_id.encode().hex()}", f"tp_rank={req.tp_rank}",
                      f"device_id={req.device_id}", f"shm={req.load_state_shm.encode().hex()}",
                      f"names={','.join(n.encode().hex() for n in req.layer_names)}",
                      f"ids={','.join(map(str, req.block_ids))}",
                      f"hashes={','.join(h.hex() for h in req.block_hashes)}"]) + "\n"


def rand_hashes(rng, n):
    return [bytes(rng.getrandbits(8) for _ in range(rng.choice([0, 1, 16, 32, 33]))) for _ in range(n)]


def test_random_requests_decode_like_the_protobuf_library(wire_test, tmp_path):
    rng = random.Random(7)
    for case in range(60):
        n = rng.choice([0, 1, 5, 300])
        shared_h, shared_ids = rand_hashes(rng, n), [rng.randint(-2**31, 2**31 - 1) for _ in range(n)]
        saves = []
        for li in range(rng.choice([0, 1, 3, 80])):
            if rng.random() < 0.7:
                ids, hs = shared_ids, shared_h
            else:
                m = rng.choice([0, 2, 7])
                ids, hs = [rng.randint(-5, 10**6) for _ in range(m)], rand_hashes(rng, m)
            saves.append(P.SaveLayer(layer_name=f"model.layers.{li}.attn-é", block_ids=ids, block_hashes=hs))
        req = P.SaveRequest(instance_id=f"inst-{case}", tp_rank=rng.choice([0, 3, 2**32 - 1]),
                            device_id=rng.choice([-1, 0, 7]), saves=saves)
        data = req.SerializeToString()
        rc, out = run(wire_test, "save", data, tmp_path)
        assert rc == 0, out
        assert out == want_save(P.SaveRequest.FromString(data)), case
        rc, out = run(wire_test, "id", data, tmp_path)
        assert out == f"instance_id={req.instance_id.encode().hex()}\n"

        lreq = P.LoadRequest(instance_id=f"i{case}", tp_rank=rng.choice([0, 5]), device_id=rng.choice([-3, 1]),
                             load_state_shm=f"pega_load_{case:032x}",
                             layer_names=[f"L{i}" for i in range(rng.choice([0, 2, 80]))],
                             block_ids=shared_ids, block_hashes=shared_h)
        data = lreq.SerializeToString()
        rc, out = run(wire_test, "load", data, tmp_path)
        assert rc == 0, out
        assert out == want_load(P.LoadRequest.FromString(data)), case


def varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def field(num: int, wt: int, payload: bytes) -> bytes:
    return varint(num << 3 | wt) + payload


def ld(num: int, data: bytes) -> bytes:
    return field(num, 2, varint(len(data)) + data)


def test_hand_written_wire_forms(wire_test, tmp_path):
    # A layer with unpacked ids, fields out of order, and unknown fields of
    # every wire type (varint, fixed64, length-delimited, fixed32).
    layer = (ld(3, b"h0") + field(2, 0, varint(5)) + field(9, 1, b"\x00" * 8) + field(2, 0, varint(-1))
             + ld(1, b"L0") + field(10, 5, b"\x00" * 4) + ld(3, b"h1") + ld(11, b"skip me"))
    data = (field(3, 0, varint(-2)) + ld(4, layer) + field(2, 0, varint(4)) + ld(1, b"first")
            + field(15, 0, varint(99)) + ld(1, b"second"))  # the last instance_id wins
    rc, out = run(wire_test, "save", data, tmp_path)
    assert rc == 0, out
    assert out == want_save(P.SaveRequest.FromString(data))
    assert "ids=5,-1 " in out and f"instance_id={b'second'.hex()}" in out
    rc, out = run(wire_test, "id", data, tmp_path)
    assert out == f"instance_id={b'second'.hex()}\n"
    # Load with packed ids split over two runs (parsers concatenate them).
    packed = ld(6, varint(1) + varint(2)) + ld(6, varint(3))
    data = ld(1, b"i") + packed + ld(7, b"a") + ld(7, b"b") + ld(7, b"c") + ld(5, b"n0")
    rc, out = run(wire_test, "load", data, tmp_path)
    assert rc == 0 and out == want_load(P.LoadRequest.FromString(data))


@pytest.mark.parametrize("data", [
    ld(1, b"abc")[:-1],                      # truncated string
    field(4, 2, varint(50)) + b"\x00" * 3,   # length past the end
    b"\xff" * 11,                            # varint longer than 10 bytes
    varint(1 << 3 | 7),                      # wire type 7 (field 1)
    varint(0),                               # field number 0
    ld(4, field(2, 2, varint(3) + b"\x80\x80\x80")),  # packed ids ending mid-varint
])
def test_malformed_requests_fail_cleanly(wire_test, tmp_path, data):
    rc, out = run(wire_test, "save", data, tmp_path)
    assert rc == 2 and out.startswith("error: invalid argument: "), out


def test_only_equal_hash_lists_are_shared(wire_test, tmp_path):
    same = [os.urandom(32) for _ in range(4)]
    other = list(same)
    other[2] = b"\x00" * 32
    req = P.SaveRequest(instance_id="i", saves=[P.SaveLayer(layer_name="a", block_ids=[1, 2, 3, 4], block_hashes=same),
                                                P.SaveLayer(layer_name="b", block_ids=[1, 2, 3, 4], block_hashes=same),
                                                P.SaveLayer(layer_name="c", block_ids=[1, 2, 3, 4], block_hashes=other),
                                                P.SaveLayer(layer_name="d", block_ids=[9], block_hashes=other)])
    rc, out = run(wire_test, "save", req.SerializeToString(), tmp_path)
    assert rc == 0
    assert [line.rsplit("shared=", 1)[1] for line in out.splitlines() if line.startswith("layer ")] == \
        ["0", "1", "0", "1"]


def test_client_encoder_matches_the_protobuf_library():
    """The client builds Save requests without a message per layer
    (encode_save_request); its bytes must be exactly the protobuf library's
    serialisation of the same request, defaults omitted, negative ids and
    device ids as ten-byte varints, layers sharing or not sharing lists."""
    from pegaflow_b200.client import encode_save_request

    rng = random.Random(3)
    for case in range(300):
        n = rng.choice([0, 1, 3, 50])
        ids = [rng.randint(-2**31, 2**31 - 1) for _ in range(n)]
        hs = [bytes(rng.getrandbits(8) for _ in range(rng.choice([0, 1, 32]))) for _ in range(n)]
        saves = []
        for li in range(rng.choice([0, 1, 2, 10])):
            if rng.random() < 0.6:
                saves.append((rng.choice(["", f"L{li}", "é" * 3]), list(ids), list(hs)))
            else:
                m = rng.choice([0, 2])
                saves.append((f"x{li}", [rng.randint(-3, 9) for _ in range(m)],
                              [bytes([li] * 4) for _ in range(m)]))
        iid, tp, dev = rng.choice(["", "inst", "ü"]), rng.choice([0, 1, 2**32 - 1]), rng.choice([-1, 0, 5, -2**31])
        want = P.SaveRequest(instance_id=iid, tp_rank=tp, device_id=dev,
                             saves=[P.SaveLayer(layer_name=a, block_ids=b, block_hashes=c) for a, b, c in saves])
        assert encode_save_request(iid, tp, dev, saves) == want.SerializeToString(), case
