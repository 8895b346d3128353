"""Message classes of the reference's gRPC schema, built at runtime.

pegaflow-proto/proto/engine.proto defines package ``pegaflow`` with seven RPCs
on service ``Engine``. protoc and grpc_tools are not available in this
environment, so the same schema — identical package, message names, field
names, numbers and types, hence the same wire format — is described here as a
FileDescriptorProto and turned into message classes by the protobuf runtime.
"""

from __future__ import annotations

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

_F = descriptor_pb2.FieldDescriptorProto
_OPT, _REP = _F.LABEL_OPTIONAL, _F.LABEL_REPEATED
_STRING, _BYTES, _BOOL = _F.TYPE_STRING, _F.TYPE_BYTES, _F.TYPE_BOOL
_I32, _U32, _U64 = _F.TYPE_INT32, _F.TYPE_UINT32, _F.TYPE_UINT64
_MSG, _ENUM = _F.TYPE_MESSAGE, _F.TYPE_ENUM

# (message, [(field, number, type, label, type_name)]) in engine.proto order.
_MESSAGES = [
    ("ResponseStatus", [("ok", 1, _BOOL, _OPT, None), ("message", 2, _STRING, _OPT, None)]),
    ("RegisterContextRequest", [
        ("instance_id", 1, _STRING, _OPT, None), ("device_id", 2, _I32, _OPT, None),
        ("layer_name", 3, _STRING, _OPT, None), ("wrapper_bytes", 4, _BYTES, _OPT, None),
        ("num_blocks", 5, _U64, _OPT, None), ("bytes_per_block", 6, _U64, _OPT, None),
        ("kv_stride_bytes", 7, _U64, _OPT, None), ("segments", 8, _U32, _OPT, None),
        ("tp_rank", 9, _U32, _OPT, None), ("tp_size", 10, _U32, _OPT, None),
        ("num_layers", 11, _U32, _OPT, None), ("namespace", 12, _STRING, _OPT, None)]),
    ("RegisterContextResponse", [("status", 1, _MSG, _OPT, ".pegaflow.ResponseStatus")]),
    ("SaveLayer", [("layer_name", 1, _STRING, _OPT, None), ("block_ids", 2, _I32, _REP, None),
                   ("block_hashes", 3, _BYTES, _REP, None)]),
    ("SaveRequest", [("instance_id", 1, _STRING, _OPT, None), ("tp_rank", 2, _U32, _OPT, None),
                     ("device_id", 3, _I32, _OPT, None), ("saves", 4, _MSG, _REP, ".pegaflow.SaveLayer")]),
    ("SaveResponse", [("status", 1, _MSG, _OPT, ".pegaflow.ResponseStatus")]),
    ("LoadRequest", [("instance_id", 1, _STRING, _OPT, None), ("tp_rank", 2, _U32, _OPT, None),
                     ("device_id", 3, _I32, _OPT, None), ("load_state_shm", 4, _STRING, _OPT, None),
                     ("layer_names", 5, _STRING, _REP, None), ("block_ids", 6, _I32, _REP, None),
                     ("block_hashes", 7, _BYTES, _REP, None)]),
    ("LoadResponse", [("status", 1, _MSG, _OPT, ".pegaflow.ResponseStatus")]),
    ("QueryRequest", [("instance_id", 1, _STRING, _OPT, None), ("block_hashes", 2, _BYTES, _REP, None)]),
    ("QueryResponse", [("status", 1, _MSG, _OPT, ".pegaflow.ResponseStatus"), ("hit_blocks", 2, _U64, _OPT, None),
                       ("prefetch_state", 3, _ENUM, _OPT, ".pegaflow.PrefetchState"),
                       ("loading_blocks", 4, _U64, _OPT, None), ("missing_blocks", 5, _U64, _OPT, None)]),
    ("UnregisterRequest", [("instance_id", 1, _STRING, _OPT, None)]),
    ("UnregisterResponse", [("status", 1, _MSG, _OPT, ".pegaflow.ResponseStatus")]),
    ("ShutdownRequest", []),
    ("ShutdownResponse", [("status", 1, _MSG, _OPT, ".pegaflow.ResponseStatus")]),
    ("HealthRequest", []),
    ("HealthResponse", [("status", 1, _MSG, _OPT, ".pegaflow.ResponseStatus")]),
]

PREFETCH_READY, PREFETCH_LOADING, PREFETCH_PARTIAL_MISS = 0, 1, 2

SERVICE = "pegaflow.Engine"
# rpc name -> (request message, response message), engine.proto:107-115
METHODS = {
    "RegisterContext": ("RegisterContextRequest", "RegisterContextResponse"),
    "Save": ("SaveRequest", "SaveResponse"),
    "Load": ("LoadRequest", "LoadResponse"),
    "Query": ("QueryRequest", "QueryResponse"),
    "UnregisterContext": ("UnregisterRequest", "UnregisterResponse"),
    "Shutdown": ("ShutdownRequest", "ShutdownResponse"),
    "Health": ("HealthRequest", "HealthResponse"),
}


def _build():
    fdp = descriptor_pb2.FileDescriptorProto()
    fdp.name = "pegaflow/engine.proto"
    fdp.package = "pegaflow"
    fdp.syntax = "proto3"
    enum = fdp.enum_type.add()
    enum.name = "PrefetchState"
    for name, num in (("PREFETCH_READY", 0), ("PREFETCH_LOADING", 1), ("PREFETCH_PARTIAL_MISS", 2)):
        v = enum.value.add()
        v.name, v.number = name, num
    for name, fields in _MESSAGES:
        m = fdp.message_type.add()
        m.name = name
        for fname, num, ftype, label, tname in fields:
            f = m.field.add()
            f.name, f.number, f.type, f.label = fname, num, ftype, label
            f.json_name = "".join(w.capitalize() if i else w for i, w in enumerate(fname.split("_")))
            if tname:
                f.type_name = tname
    svc = fdp.service.add()
    svc.name = "Engine"
    for rpc, (req, resp) in METHODS.items():
        md = svc.method.add()
        md.name, md.input_type, md.output_type = rpc, f".pegaflow.{req}", f".pegaflow.{resp}"
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fdp)
    return {name: message_factory.GetMessageClass(pool.FindMessageTypeByName(f"pegaflow.{name}"))
            for name, _ in _MESSAGES}


M = _build()
globals().update(M)
