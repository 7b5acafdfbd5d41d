"""CPU tests of the C ABI: the library loads, exports exactly what include/onnxb200.h
declares, and its host-only entry points (shape inference, status strings) agree
with the oracle.  No kernel is launched."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "onnxb200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"ONNXB200_API\s+[\w\s\*]+?\b(onnxb200_\w+)\s*\(", src)))


def test_library_loads_and_exports_header(ob):
    lib = ob._capi.lib()
    decl = declared_symbols()
    assert len(decl) >= 30
    for name in decl:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", ob.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(l.split()[-1] for l in out.splitlines() if " T " in l)
    assert exported == decl
    assert set(ob._capi.SIGNATURES) == set(decl)


def test_version_and_status_strings(ob):
    lib = ob._capi.lib()
    assert lib.onnxb200_version() >= 100
    assert lib.onnxb200_status_string(0) == b"ok"
    assert lib.onnxb200_status_string(4) == b"operation timed out"
    assert lib.onnxb200_last_error(None) == b"null handle"


def test_null_arguments_rejected(ob):
    lib = ob._capi.lib()
    assert lib.onnxb200_create(0, None, None) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_destroy(None) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_synchronize(None) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_graph_destroy(None) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_graph_run_host_pipelined(None, None, 1, None, None) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_graph_build_from_model(None, None, None, 0, None) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_conv_nd(None, None, None, None, None, None) == ob._capi.ERR_INVALID_ARGUMENT
    p = ctypes.c_void_p()
    assert lib.onnxb200_malloc(None, 16, ctypes.byref(p)) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_free(None, None) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_memcpy(None, None, None, 16, 0) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_model_parse(None, 0, None, None, None, 0) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_model_load(None, None, None, 0) == ob._capi.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_model_destroy(None) == ob._capi.OK
    assert lib.onnxb200_status_string(ob._capi.ERR_PROTOBUF) == b"protobuf parsing error"


@pytest.mark.parametrize("cfg", [
    # x shape, w shape, strides, pads, dilations, group, auto_pad
    ((1, 3, 224, 224), (64, 3, 7, 7), (2, 2), (3, 3, 3, 3), (1, 1), 1, "NOTSET"),
    ((1, 1, 5, 5), (1, 1, 2, 2), (1, 1), (0, 0, 0, 0), (2, 2), 1, "NOTSET"),
    ((1, 1, 5, 5), (1, 1, 2, 2), (2, 2), (0, 0, 0, 0), (1, 1), 1, "NOTSET"),
    ((1, 1, 3, 3), (1, 1, 3, 3), (1, 1), (0, 0, 0, 0), (1, 1), 1, "SAME_UPPER"),
    ((1, 1, 3, 3), (1, 1, 3, 3), (1, 1), (0, 0, 0, 0), (1, 1), 1, "VALID"),
    ((2, 128, 28, 28), (128, 4, 3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 32, "NOTSET"),
    ((2, 256, 28, 28), (256, 256, 3, 3), (1, 1), (2, 2, 2, 2), (2, 2), 1, "NOTSET"),
    ((3, 8, 224, 224), (16, 8, 7, 7), (2, 2), (0, 0, 0, 0), (1, 1), 1, "SAME_LOWER"),
])
def test_conv_output_shape_matches_oracle(ob, oracle, cfg):
    xs, ws, st, pd, dl, g, ap = cfg
    conv = ob.Conv(st, pd, dl, g, ap)
    shape = conv.output_shape(xs, ws)
    if ap in ("SAME_UPPER", "SAME_LOWER"):
        up = ap == "SAME_UPPER"
        pt, pb = oracle.same_pads(xs[2], ws[2], st[0], dl[0], up)
        pl, pr = oracle.same_pads(xs[3], ws[3], st[1], dl[1], up)
    elif ap == "VALID":
        pt = pl = pb = pr = 0
    else:
        pt, pl, pb, pr = pd
    exp = [xs[0], ws[0], oracle.conv_out_dim(xs[2], ws[2], st[0], pt, pb, dl[0]),
           oracle.conv_out_dim(xs[3], ws[3], st[1], pl, pr, dl[1])]
    assert shape == exp


@pytest.mark.parametrize("cfg", [
    # x shape, w shape, strides, pads, dilations, group, auto_pad
    ((1, 1, 5), (1, 1, 3), None, None, None, 1, "NOTSET"),
    ((2, 4, 17), (6, 2, 5), (2,), (2, 1), (1,), 2, "NOTSET"),
    ((2, 3, 16), (8, 3, 4), (3,), None, (2,), 1, "SAME_UPPER"),
    ((1, 2, 9), (4, 2, 3), (2,), None, None, 1, "SAME_LOWER"),
    ((1, 1, 2, 2, 2), (1, 1, 2, 2, 2), None, None, None, 1, "NOTSET"),
    ((2, 4, 7, 9, 8), (6, 2, 3, 3, 2), (2, 1, 2), (1, 0, 1, 1, 2, 0), (1, 2, 1), 2, "NOTSET"),
    ((1, 3, 8, 8, 8), (5, 3, 3, 3, 3), (2, 2, 2), None, None, 1, "SAME_UPPER"),
])
def test_conv_nd_output_shape_matches_oracle(ob, oracle, cfg):
    """1-D and 3-D Conv::output_shapes (conv.rs:205-323) against the oracle's
    shape rules (the oracle evaluates the same convolution directly)."""
    xs, ws, st, pd, dl, g, ap = cfg
    sp = len(xs) - 2
    shape = ob.Conv(st, pd, dl, g, ap).output_shape(xs, ws)
    st = st or [1] * sp
    dl = dl or [1] * sp
    if ap in ("SAME_UPPER", "SAME_LOWER"):
        ps = [oracle.same_pads(xs[2 + i], ws[2 + i], st[i], dl[i], ap == "SAME_UPPER") for i in range(sp)]
        pb, pe = [p[0] for p in ps], [p[1] for p in ps]
    else:
        pd = pd or [0] * (2 * sp)
        pb, pe = pd[:sp], pd[sp:]
    exp = [xs[0], ws[0]] + [oracle.conv_out_dim(xs[2 + i], ws[2 + i], st[i], pb[i], pe[i], dl[i])
                            for i in range(sp)]
    assert shape == exp
    if ap == "NOTSET":  # the oracle's direct convolution produces that shape
        x = np.zeros(xs, np.float32)
        w = np.zeros(ws, np.float32)
        assert list(oracle.conv_nd_direct(x, w, None, st, pb + pe, dl, g).shape) == exp


def test_conv_nd_rejects_bad_attributes(ob):
    with pytest.raises(ob.ValidationError):
        ob.Conv((1, 1), None, None).output_shape((1, 2, 8), (3, 2, 3))  # 2 strides for 1 spatial dim
    with pytest.raises(ob.ValidationError):
        ob.Conv().output_shape((1, 2, 2, 2, 2, 2), (1, 2, 1, 1, 1, 1))  # 4 spatial dims
    with pytest.raises(ob.ValidationError):
        ob.Conv(group=3).output_shape((1, 8, 5), (4, 2, 3))


def test_conv_output_shape_rejects_bad_groups(ob):
    with pytest.raises(ob.ValidationError):
        ob.Conv(group=3).output_shape((1, 8, 5, 5), (4, 2, 3, 3))


def test_matmul_output_shape_matches_oracle(ob, oracle):
    cases = [((2, 3), (3, 4)), ((3,), (3,)), ((3,), (3, 2)), ((2, 3), (3,)), ((2, 3, 4), (2, 4, 5)),
             ((2, 1, 3, 4), (2, 5, 4, 5)), ((3, 4), (2, 4, 5)), ((8, 1, 512, 768), (12, 768, 3072))]
    for a, b in cases:
        assert ob.MatMul.output_shape(a, b) == oracle.matmul_shape(a, b)
    for a, b in [((2, 3), (4, 5)), ((2,), (3,)), ((2, 3, 4), (3, 4, 5)), ((5, 10, 20), (10, 20, 30))]:
        with pytest.raises(ob.ValidationError):
            ob.MatMul.output_shape(a, b)


def test_registry_resolves_versions(ob):
    r = ob.OperatorRegistry.initialize_standard_operators()
    op = r.create_operator_for_node({"op": "Conv", "inputs": ["x", "w"], "outputs": ["y"],
                                     "attrs": {"strides": [2, 2], "pads": [3, 3, 3, 3]}}, opset=13)
    assert isinstance(op, ob.Conv) and op.strides == [2, 2] and op.pads == [3, 3, 3, 3]
    with pytest.raises(ob.InvalidOperator):
        r.create_operator_for_node({"op": "Conv", "inputs": [], "outputs": []}, opset=10)
    with pytest.raises(ob.InvalidOperator):
        r.create_operator_for_node({"op": "Softmax", "inputs": [], "outputs": []})
    with pytest.raises(ob.InvalidOperator):
        r.register_operator("Conv", "", 11, ob.Conv)
    mp = r.create_operator_for_node({"op": "MaxPool", "attrs": {"kernel_shape": [3, 3], "strides": [2, 2],
                                                                "pads": [1, 1, 1, 1]}})
    assert mp.output_shapes({"attrs": {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]}},
                            [[2, 64, 112, 112]]) == [[2, 64, 56, 56]]


def test_synth_is_deterministic(ob):
    a = ob.synth.normal(4, "X", (3, 5))
    b = ob.synth.normal(4, "X", (3, 5))
    c = ob.synth.normal(4, "Y", (3, 5))
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, c)
    u = ob.synth.uniform(0, "X", (10000,), -1, 1)
    assert u.min() >= -1 and u.max() < 1 and abs(u.mean()) < 0.05
    n = ob.synth.normal(1, "A", (100000,))
    assert abs(n.mean()) < 0.02 and abs(n.std() - 1) < 0.02


def test_workload_graphs_are_well_formed(ob):
    for build in (ob.workloads.resnet18, ob.workloads.resnet50):
        nodes, inits, ins, outs = build(batch=2)
        produced = {n["outputs"][0] for n in nodes}
        for n in nodes:
            for i in n["inputs"]:
                assert i in produced or i in inits or i == ins[0][0], i
        assert outs[0] in produced
    nodes, _, _, _ = ob.workloads.resnet50(batch=1)
    assert sum(1 for n in nodes if n["op"] == "Conv") == 53
    # 4.09 GMAC per image for ResNet-50 v1.5 convolutions
    assert abs(ob.workloads.resnet50.conv_flops_per_image / 2 - 4.09e9) / 4.09e9 < 0.02
    nodes, _, _, _ = ob.workloads.resnet18(batch=1)
    assert sum(1 for n in nodes if n["op"] == "Conv") == 20


def test_infer_shapes_matches_oracle(ob, oracle):
    """onnxb200_infer_shapes gives every node output's shape of ResNet-18 (node
    list, no graph, no GPU) equal to the shape the oracle computes."""
    nodes, inits, ins, outs = ob.workloads.resnet18(batch=1, seed=2)
    known = {k: list(v.shape) for k, v in inits.items()}
    known.update({n: s for n, s in ins})
    shapes = ob.infer_shapes(nodes, known)
    names = [o for nd in nodes for o in nd["outputs"]]
    assert list(shapes) == names
    ref = oracle.run_graph(nodes, inits, {"X": ob.workloads.resnet_input(2, 1)}, names)
    for n in names:
        assert shapes[n] == list(ref[n].shape), n
    assert shapes["logits"] == [1, 1000]
    # a batch of 256 without building anything
    known["X"] = [256, 3, 224, 224]
    assert ob.infer_shapes(nodes, known)["logits"] == [256, 1000]


def test_infer_shapes_errors(ob):
    C = ob._capi
    conv = {"op": "Conv", "inputs": ["X", "W"], "outputs": ["Y"], "attrs": {"pads": [1, 1, 1, 1]}}
    with pytest.raises(ob.ValidationError):  # channel mismatch
        ob.infer_shapes([conv], {"X": [1, 8, 5, 5], "W": [4, 3, 3, 3]})
    with pytest.raises(ob.InvalidOperator):
        ob.infer_shapes([{"op": "Softmax", "inputs": ["X"], "outputs": ["Y"]}], {"X": [2, 3]})
    with pytest.raises(ob.InvalidGraph):  # input without a producer or a shape
        ob.infer_shapes([conv], {"W": [4, 8, 3, 3]})
    assert ob.infer_shapes([conv], {"X": [2, 8, 5, 5], "W": [4, 8, 3, 3]}) == {"Y": [2, 4, 5, 5]}
    n = ctypes.c_int()
    assert C.lib().onnxb200_infer_shapes(None, 0, None, 0, None, 0, None, None, 0) == C.ERR_INVALID_ARGUMENT
    assert C.lib().onnxb200_infer_shapes(None, 0, None, 0, None, 0, ctypes.byref(n), None, 0) == C.OK
    assert n.value == 0


def test_multi_build_argument_checks(ob):
    """The multi-device build rejects bad arguments before touching a GPU."""
    C = ob._capi
    lib = C.lib()
    p = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    assert lib.onnxb200_multi_build(None, 0, None, None, 0, None, 0, None, 0, None, 0, ctypes.byref(p), err,
                                    256) == C.ERR_INVALID_ARGUMENT
    with pytest.raises(ob.ValidationError, match="fewer images than devices"):
        ob.MultiGraph([0, 1, 2], [{"op": "Relu", "inputs": ["X"], "outputs": ["Y"]}], {}, [("X", [2, 4])], ["Y"])
    with pytest.raises(ob.ValidationError, match="listed twice"):
        ob.MultiGraph([0, 0], [{"op": "Relu", "inputs": ["X"], "outputs": ["Y"]}], {}, [("X", [2, 4])], ["Y"])
    with pytest.raises(ob.ValidationError, match="disagree"):
        ob.MultiGraph([0], [{"op": "Add", "inputs": ["X", "Z"], "outputs": ["Y"]}], {},
                      [("X", [2, 4]), ("Z", [3, 4])], ["Y"])
    assert lib.onnxb200_multi_run_host(None, 1, None, None) == C.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_multi_destroy(None) == C.ERR_INVALID_ARGUMENT
    assert lib.onnxb200_multi_last_error(None) == b"null multi-device graph"
