"""ONNX ModelProto reader (onnxb200_model_parse / _load) and the test-graph writer.

The checker here is an independent protobuf implementation: the installed
google.protobuf runtime, given message descriptors with the field numbers of
the reference's proto/onnx.proto:65-470 (TensorProto's external data in the
standard ONNX form), decodes what the writer encodes and encodes models the
library's reader must parse.  The reader follows OnnxModelLoader
(src/parser/model_loader.rs:27-454).  No GPU is needed.
"""
import numpy as np
import pytest

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

_F = descriptor_pb2.FieldDescriptorProto
_I64, _I32, _FLT, _STR, _BYTES, _MSG = _F.TYPE_INT64, _F.TYPE_INT32, _F.TYPE_FLOAT, _F.TYPE_STRING, _F.TYPE_BYTES, _F.TYPE_MESSAGE
_OPT, _REP = _F.LABEL_OPTIONAL, _F.LABEL_REPEATED

# message -> [(field, number, type, label, message type, packed)]
_SCHEMA = {
    "StringStringEntryProto": [("key", 1, _STR, _OPT, None, False), ("value", 2, _STR, _OPT, None, False)],
    "OperatorSetIdProto": [("domain", 1, _STR, _OPT, None, False), ("version", 2, _I64, _OPT, None, False)],
    "Dimension": [("dim_value", 1, _I64, _OPT, None, False), ("dim_param", 2, _STR, _OPT, None, False)],
    "TensorShapeProto": [("dim", 1, _MSG, _REP, "Dimension", False)],
    "TypeProtoTensor": [("elem_type", 1, _I32, _OPT, None, False), ("shape", 2, _MSG, _OPT, "TensorShapeProto", False)],
    "TypeProto": [("tensor_type", 1, _MSG, _OPT, "TypeProtoTensor", False)],
    "ValueInfoProto": [("name", 1, _STR, _OPT, None, False), ("type", 2, _MSG, _OPT, "TypeProto", False)],
    "TensorProto": [("dims", 1, _I64, _REP, None, False), ("data_type", 2, _I32, _OPT, None, False),
                    ("float_data", 4, _FLT, _REP, None, True), ("int64_data", 7, _I64, _REP, None, True),
                    ("name", 8, _STR, _OPT, None, False), ("raw_data", 9, _BYTES, _OPT, None, False),
                    ("external_data", 13, _MSG, _REP, "StringStringEntryProto", False),
                    ("data_location", 14, _I32, _OPT, None, False)],
    "AttributeProto": [("name", 1, _STR, _OPT, None, False), ("f", 2, _FLT, _OPT, None, False),
                       ("i", 3, _I64, _OPT, None, False), ("s", 4, _BYTES, _OPT, None, False),
                       ("t", 5, _MSG, _OPT, "TensorProto", False), ("floats", 7, _FLT, _REP, None, False),
                       ("ints", 8, _I64, _REP, None, False), ("type", 20, _I32, _OPT, None, False)],
    "NodeProto": [("input", 1, _STR, _REP, None, False), ("output", 2, _STR, _REP, None, False),
                  ("name", 3, _STR, _OPT, None, False), ("op_type", 4, _STR, _OPT, None, False),
                  ("attribute", 5, _MSG, _REP, "AttributeProto", False), ("domain", 7, _STR, _OPT, None, False)],
    "GraphProto": [("node", 1, _MSG, _REP, "NodeProto", False), ("name", 2, _STR, _OPT, None, False),
                   ("initializer", 5, _MSG, _REP, "TensorProto", False),
                   ("input", 11, _MSG, _REP, "ValueInfoProto", False),
                   ("output", 12, _MSG, _REP, "ValueInfoProto", False),
                   ("value_info", 13, _MSG, _REP, "ValueInfoProto", False)],
    "ModelProto": [("ir_version", 1, _I64, _OPT, None, False), ("producer_name", 2, _STR, _OPT, None, False),
                   ("graph", 7, _MSG, _OPT, "GraphProto", False),
                   ("opset_import", 8, _MSG, _REP, "OperatorSetIdProto", False)],
}


@pytest.fixture(scope="module")
def pb():
    fd = descriptor_pb2.FileDescriptorProto(name="onnx_subset_test.proto", package="onnxsub", syntax="proto2")
    for mname, fields in _SCHEMA.items():
        m = fd.message_type.add(name=mname)
        for fname, num, ftype, label, tname, packed in fields:
            f = m.field.add(name=fname, number=num, type=ftype, label=label)
            if tname:
                f.type_name = ".onnxsub." + tname
            if packed:
                f.options.packed = True
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    return {n: message_factory.GetMessageClass(pool.FindMessageTypeByName("onnxsub." + n)) for n in _SCHEMA}


@pytest.fixture(scope="module")
def r18(ob):
    return ob.workloads.resnet18(batch=1, seed=2)


def test_roundtrip_resnet18(ob, r18):
    nodes, inits, ins, outs = r18
    m = ob.onnx_io.load(ob.onnx_io.encode_model(nodes, inits, ins, outs, opset=13))
    assert m.info["opset"] == 13 and m.info["ir_version"] == 8
    assert m.info["n_skipped_initializers"] == 0 and m.info["n_skipped_attributes"] == 0
    def norm(v):  # ONNX FLOAT attributes are fp32
        return list(v) if isinstance(v, (list, tuple)) else float(np.float32(v)) if isinstance(v, float) else v

    assert m.nodes == [{"op": n["op"], "inputs": list(n["inputs"]), "outputs": list(n["outputs"]),
                        "attrs": {k: norm(v) for k, v in n.get("attrs", {}).items()}} for n in nodes]
    got = m.initializers
    assert list(got) == list(inits)
    for k, v in inits.items():
        assert got[k].shape == np.asarray(v).shape
        assert got[k].tobytes() == np.ascontiguousarray(v, np.float32).tobytes()
    assert m.inputs == [(n, list(s)) for n, s in ins]
    assert m.outputs == list(outs)


def test_protobuf_runtime_decodes_writer(ob, pb, r18):
    nodes, inits, ins, outs = r18
    model = pb["ModelProto"]()
    model.ParseFromString(ob.onnx_io.encode_model(nodes, inits, ins, outs, opset=17, graph_name="r18"))
    assert model.ir_version == 8 and model.opset_import[0].version == 17 and model.opset_import[0].domain == ""
    g = model.graph
    assert g.name == "r18" and len(g.node) == len(nodes)
    for pn, nd in zip(g.node, nodes):
        assert pn.op_type == nd["op"] and list(pn.input) == list(nd["inputs"]) and list(pn.output) == list(nd["outputs"])
        for a in pn.attribute:
            v = nd["attrs"][a.name]
            if a.type == 7:
                assert list(a.ints) == list(v)
            elif a.type == 2:
                assert a.i == v
            elif a.type == 1:
                assert np.float32(a.f) == np.float32(v)
            else:
                assert a.type == 3 and a.s.decode() == v
    for t in g.initializer:
        assert t.data_type == 1
        assert t.raw_data == np.ascontiguousarray(inits[t.name], np.float32).tobytes()
        assert list(t.dims) == list(np.asarray(inits[t.name]).shape)
    assert [(v.name, [d.dim_value for d in v.type.tensor_type.shape.dim]) for v in g.input] == \
        [(n, list(s)) for n, s in ins]


def _vi(pb, name, dims):
    v = pb["ValueInfoProto"](name=name)
    v.type.tensor_type.elem_type = 1
    for d in dims:
        dim = v.type.tensor_type.shape.dim.add()
        if isinstance(d, str):
            dim.dim_param = d
        else:
            dim.dim_value = d
    return v


def _small_model(pb, rng):
    """Conv(+bias) -> Relu -> GlobalAveragePool -> Flatten -> Gemm, encoded by
    the protobuf runtime: float_data instead of raw_data, graph inputs that list
    the initializers (IR version 3 style), a symbolic batch dimension, an
    int64 initializer and attribute kinds the reader skips."""
    w = rng.standard_normal((8, 4, 3, 3)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    fw = rng.standard_normal((5, 8)).astype(np.float32)
    fb = rng.standard_normal(5).astype(np.float32)
    m = pb["ModelProto"](ir_version=3, producer_name="pb-runtime")
    m.opset_import.add(domain="ai.onnx", version=11)
    m.opset_import.add(domain="com.example", version=2)
    g = m.graph
    g.name = "small"
    for name, arr in (("w", w), ("b", b), ("fw", fw), ("fb", fb)):
        t = g.initializer.add(name=name, data_type=1)
        t.dims.extend(arr.shape)
        t.float_data.extend(arr.ravel().tolist())
    shape_const = g.initializer.add(name="shape_const", data_type=7)
    shape_const.dims.append(2)
    shape_const.int64_data.extend([1, -1])
    g.input.extend([_vi(pb, "X", ["N", 4, 6, 6])] + [_vi(pb, n, a.shape) for n, a in (("w", w), ("b", b), ("fw", fw), ("fb", fb))])
    g.output.append(_vi(pb, "Y", ["N", 5]))
    conv = g.node.add(op_type="Conv", name="conv")
    conv.input.extend(["X", "w", "b"])
    conv.output.append("c")
    for k, v in (("kernel_shape", [3, 3]), ("pads", [1, 1, 1, 1]), ("strides", [1, 1])):
        a = conv.attribute.add(name=k, type=7)
        a.ints.extend(v)
    a = conv.attribute.add(name="auto_pad", type=3, s=b"NOTSET")
    a = conv.attribute.add(name="unused_floats", type=6)
    a.floats.extend([0.5, 1.5])
    a = conv.attribute.add(name="unused_tensor", type=4)
    a.t.data_type = 1
    a.t.float_data.append(2.0)
    relu = g.node.add(op_type="Relu", input=["c"], output=["r"])
    gap = g.node.add(op_type="GlobalAveragePool", input=["r"], output=["p"])
    flat = g.node.add(op_type="Flatten", input=["p"], output=["f"])
    flat.attribute.add(name="axis", type=2, i=1)
    gemm = g.node.add(op_type="Gemm", input=["f", "fw", "fb"], output=["Y"])
    gemm.attribute.add(name="transB", type=2, i=1)
    gemm.attribute.add(name="alpha", type=1, f=0.75)
    del relu, gap
    return m, {"w": w, "b": b, "fw": fw, "fb": fb}


def test_reader_parses_protobuf_runtime_model(ob, pb, oracle):
    m_pb, weights = _small_model(pb, np.random.default_rng(7))
    m = ob.onnx_io.load(m_pb.SerializeToString())
    info = m.info
    assert info["ir_version"] == 3 and info["opset"] == 11 and info["producer_name"] == "pb-runtime"
    assert info["graph_name"] == "small"
    assert info["n_skipped_initializers"] == 1 and info["n_skipped_attributes"] == 2
    assert m.inputs == [("X", [-1, 4, 6, 6])]  # initializers are not inputs; "N" is symbolic
    assert m.outputs == ["Y"]
    inits = m.initializers
    assert set(inits) == set(weights)
    for k, v in weights.items():
        assert inits[k].tobytes() == v.tobytes() and inits[k].shape == v.shape
    nodes = m.nodes
    assert [n["op"] for n in nodes] == ["Conv", "Relu", "GlobalAveragePool", "Flatten", "Gemm"]
    assert nodes[0]["attrs"] == {"kernel_shape": [3, 3], "pads": [1, 1, 1, 1], "strides": [1, 1],
                                 "auto_pad": "NOTSET"}
    assert nodes[3]["attrs"] == {"axis": 1}
    assert nodes[4]["attrs"] == {"transB": 1, "alpha": 0.75}
    # the parsed graph computes what the protobuf runtime's graph describes
    x = np.random.default_rng(8).standard_normal((2, 4, 6, 6)).astype(np.float32)
    ref_nodes = [{"op": n.op_type, "inputs": list(n.input), "outputs": list(n.output),
                  "attrs": {"kernel_shape": [3, 3], "pads": [1, 1, 1, 1], "strides": [1, 1]} if n.op_type == "Conv"
                  else {"axis": 1} if n.op_type == "Flatten" else {"transB": 1, "alpha": 0.75} if n.op_type == "Gemm"
                  else {}} for n in m_pb.graph.node]
    y = oracle.run_graph(nodes, inits, {"X": x}, ["Y"])["Y"]
    y_ref = oracle.run_graph(ref_nodes, weights, {"X": x}, ["Y"])["Y"]
    assert y.shape == (2, 5) and np.array_equal(y, y_ref)


def test_reader_packed_and_unpacked_repeated_fields(ob):
    io = ob.onnx_io
    # Conv attribute "pads" packed (one length-delimited run), "strides" unpacked
    packed = io._key(8, 2) + io._varint(4) + bytes([1, 1, 1, 1])
    attr_p = io._str(1, "pads") + packed + io._int(20, 7)
    attr_u = io._attribute("strides", [2, 2])
    node = io._str(1, "X") + io._str(1, "W") + io._str(2, "Y") + io._str(4, "Conv") + io._ld(5, attr_p) + io._ld(5, attr_u)
    w = np.arange(2 * 3 * 3 * 3, dtype=np.float32).reshape(2, 3, 3, 3)
    # weights as unpacked float_data entries (one fixed32 each); dims packed
    t = io._ld(1, b"".join(io._varint(d) for d in w.shape)) + io._int(2, 1) + io._str(8, "W")
    t += b"".join(io._float(4, float(v)) for v in w.ravel())
    g = io._ld(1, node) + io._ld(5, t) + io._ld(11, io._value_info("X", [1, 3, 8, 8])) + io._ld(12, io._value_info("Y", None))
    m = io.load(io._int(1, 7) + io._ld(7, g))
    assert m.nodes[0]["attrs"] == {"pads": [1, 1, 1, 1], "strides": [2, 2]}
    assert m.initializers["W"].tobytes() == w.tobytes()
    assert m.info["opset"] == 1  # no opset import: the default domain starts at version 1


def test_reader_errors(ob, tmp_path):
    io = ob.onnx_io
    nodes, inits, ins, outs = ob.workloads.stem_conv(seed=0)
    good = io.encode_model(nodes, inits, ins, outs)
    with pytest.raises(ob.ProtobufError):
        io.load(good[: len(good) // 2])  # truncated
    with pytest.raises(ob.ProtobufError):
        io.load(io._key(7, 0) + io._varint(5))  # graph field with a varint wire type
    with pytest.raises(ob.InvalidModel):
        io.load(io._int(1, 8))  # no graph
    bad_attr = io._ld(7, io._ld(1, io._str(4, "Relu") + io._ld(5, io._str(1, "x") + io._int(3, 1))))
    with pytest.raises(ob.InvalidModel):
        io.load(bad_attr)  # attribute without a type
    bad_raw = io._ld(7, io._ld(5, io._int(1, 4) + io._int(2, 1) + io._str(8, "t") + io._ld(9, b"\0" * 12)))
    with pytest.raises(ob.InvalidModel):
        io.load(bad_raw)  # raw_data of 3 floats for a [4] tensor
    no_type = io._ld(7, io._ld(11, io._str(1, "X")))
    with pytest.raises(ob.InvalidModel):
        io.load(no_type)  # graph input without a type
    ext = io.encode_model(nodes, inits, ins, outs, external=("w.data", []))
    with pytest.raises(ob.UnsupportedFeature):
        io.load(ext)  # external data from memory, no base directory
    with pytest.raises(ob.IoError):
        io.load(str(tmp_path / "missing.onnx"))
    with pytest.raises(ob.IoError):
        io.load(ext, base_dir=str(tmp_path))  # w.data does not exist
    escape = io._ld(7, io._ld(5, io._int(1, 1) + io._int(2, 1) + io._str(8, "t")
                              + io._ld(13, io._str(1, "location") + io._str(2, "../secret")) + io._int(14, 1)))
    with pytest.raises(ob.InvalidModel):
        io.load(escape, base_dir=str(tmp_path))


def test_external_data_file(ob, tmp_path, r18):
    nodes, inits, ins, outs = r18
    path = str(tmp_path / "r18.onnx")
    ob.onnx_io.save(path, nodes, inits, ins, outs, external_data=True)
    import os
    assert os.path.getsize(path) < 64 * 1024  # weights are in r18.onnx.data
    m = ob.onnx_io.load(path)
    got = m.initializers
    for k, v in inits.items():
        assert got[k].tobytes() == np.ascontiguousarray(v, np.float32).tobytes()
    assert len(m.nodes) == len(nodes)
