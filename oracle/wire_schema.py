"""mlvc.wire schema built at run time with the protobuf library.

TEST INFRASTRUCTURE ONLY.  The reference serialises AOT graphs with the
proto3 schema in proto/mlvc_model.proto:1-83 (Graph, Node, TensorDescriptor,
ConvAttributes, ...).  No protoc is available, so this module declares the
same field numbers and types through descriptor_pb2 and lets the protobuf
runtime parse graph.pb files.  It is an independent decoder against which the
product's own wire reader (mlvc_b200.graph / csrc/host/wire.cpp) is checked.
"""

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

_F = descriptor_pb2.FieldDescriptorProto


def _field(msg, name, number, ftype, label=_F.LABEL_OPTIONAL, type_name=None, oneof=None, packed=None):
    f = msg.field.add(name=name, number=number, type=ftype, label=label)
    if type_name:
        f.type_name = type_name
    if oneof is not None:
        f.oneof_index = oneof
    return f


def _build():
    fd = descriptor_pb2.FileDescriptorProto(name="mlvc_wire_oracle.proto", package="mlvc.wire", syntax="proto3")
    dt = fd.enum_type.add(name="DataType")
    for n, v in (("DATA_TYPE_UNSPECIFIED", 0), ("FP16", 1), ("INT32", 2), ("INT64", 3)):
        dt.value.add(name=n, number=v)
    ok = fd.enum_type.add(name="OpKind")
    for v, n in enumerate(("OP_UNSPECIFIED", "ADD", "SUB", "MUL", "CLIP", "CONCAT", "CONV", "DEPTH_TO_SPACE",
                           "GATHER", "LEAKY_RELU", "RECIPROCAL", "ROUND", "SIGMOID", "SLICE", "SPACE_TO_DEPTH")):
        ok.value.add(name=n, number=v)
    R = _F.LABEL_REPEATED
    m = fd.message_type.add(name="ConvAttributes")
    _field(m, "strides", 1, _F.TYPE_UINT32, R)
    _field(m, "pads", 2, _F.TYPE_UINT32, R)
    _field(m, "dilations", 3, _F.TYPE_UINT32, R)
    _field(m, "groups", 4, _F.TYPE_UINT32)
    m = fd.message_type.add(name="AxisAttributes")
    _field(m, "axis", 1, _F.TYPE_SINT32)
    m = fd.message_type.add(name="ActivationAttributes")
    _field(m, "alpha", 1, _F.TYPE_FLOAT)
    m = fd.message_type.add(name="PixelAttributes")
    _field(m, "block_size", 1, _F.TYPE_UINT32)
    m = fd.message_type.add(name="Node")
    m.oneof_decl.add(name="attributes")
    _field(m, "op", 1, _F.TYPE_ENUM, type_name=".mlvc.wire.OpKind")
    _field(m, "inputs", 2, _F.TYPE_UINT32, R)
    _field(m, "outputs", 3, _F.TYPE_UINT32, R)
    _field(m, "conv", 4, _F.TYPE_MESSAGE, type_name=".mlvc.wire.ConvAttributes", oneof=0)
    _field(m, "axis", 5, _F.TYPE_MESSAGE, type_name=".mlvc.wire.AxisAttributes", oneof=0)
    _field(m, "activation", 6, _F.TYPE_MESSAGE, type_name=".mlvc.wire.ActivationAttributes", oneof=0)
    _field(m, "pixel", 7, _F.TYPE_MESSAGE, type_name=".mlvc.wire.PixelAttributes", oneof=0)
    m = fd.message_type.add(name="ArenaAllocation")
    _field(m, "offset", 1, _F.TYPE_UINT64)
    _field(m, "size_bytes", 2, _F.TYPE_UINT64)
    _field(m, "birth", 3, _F.TYPE_UINT32)
    _field(m, "death", 4, _F.TYPE_UINT32)
    m = fd.message_type.add(name="WeightLocation")
    _field(m, "offset", 1, _F.TYPE_UINT64)
    _field(m, "size_bytes", 2, _F.TYPE_UINT64)
    m = fd.message_type.add(name="TensorDescriptor")
    m.oneof_decl.add(name="storage")
    _field(m, "id", 1, _F.TYPE_UINT32)
    _field(m, "name", 2, _F.TYPE_STRING)
    _field(m, "dtype", 3, _F.TYPE_ENUM, type_name=".mlvc.wire.DataType")
    _field(m, "shape", 4, _F.TYPE_INT64, R)
    _field(m, "arena", 5, _F.TYPE_MESSAGE, type_name=".mlvc.wire.ArenaAllocation", oneof=0)
    _field(m, "weight", 6, _F.TYPE_MESSAGE, type_name=".mlvc.wire.WeightLocation", oneof=0)
    m = fd.message_type.add(name="Graph")
    _field(m, "schema_version", 1, _F.TYPE_UINT32)
    _field(m, "checkpoint_sha256", 2, _F.TYPE_BYTES)
    _field(m, "tensors", 3, _F.TYPE_MESSAGE, R, type_name=".mlvc.wire.TensorDescriptor")
    _field(m, "inputs", 4, _F.TYPE_UINT32, R)
    _field(m, "outputs", 5, _F.TYPE_UINT32, R)
    _field(m, "nodes", 6, _F.TYPE_MESSAGE, R, type_name=".mlvc.wire.Node")
    _field(m, "arena_bytes", 7, _F.TYPE_UINT64)
    _field(m, "arena_alignment", 8, _F.TYPE_UINT32)
    _field(m, "weights_bytes", 9, _F.TYPE_UINT64)
    _field(m, "weights_sha256", 10, _F.TYPE_BYTES)
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    return message_factory.GetMessageClass(pool.FindMessageTypeByName("mlvc.wire.Graph"))


Graph = _build()

OP_NAMES = {1: "Add", 2: "Sub", 3: "Mul", 4: "Clip", 5: "Concat", 6: "Conv", 7: "DepthToSpace", 8: "Gather",
            9: "LeakyRelu", 10: "Reciprocal", 11: "Round", 12: "Sigmoid", 13: "Slice", 14: "SpaceToDepth"}


def parse_graph(data: bytes):
    g = Graph()
    g.ParseFromString(data)
    return g
