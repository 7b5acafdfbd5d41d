"""GPU end-to-end tests of the graph executor against the oracle evaluating the
same unfused node list node by node.

End-to-end logits: an element passes if |a-b| <= 1e-3 * max|ref| or
|a-b|/|b| <= 1e-3 (3xTF32); 2e-2 for the tf32 / bf16 fast modes.  The absolute
term is scaled by the logits' magnitude because the randomly initialised
networks (BatchNormalization gamma = 1 everywhere) grow activations to ~1e4.
"""
import importlib

import numpy as np
import pytest
import torch

from conftest import compare

pytestmark = pytest.mark.gpu

ob_mod = importlib.import_module("onnx-rs_b200")


def check_logits(y, ref, tol, what):
    scale = float(np.abs(ref).max())
    n, ma, mr = compare(y, ref, tol, tol * scale)
    assert n == 0, f"{what}: {n} logits outside tolerance (max abs {ma:.3g} vs scale {scale:.3g}, max rel {mr:.3g})"
    return ma / scale


@pytest.fixture(scope="module")
def r18_ref(oracle):
    nodes, inits, ins, outs = ob_mod.workloads.resnet18(batch=2, seed=2)
    x = ob_mod.workloads.resnet_input(2, 2)
    ref = oracle.run_graph(nodes, inits, {"X": x}, outs)[outs[0]]
    return nodes, inits, ins, outs, x, ref


@pytest.mark.parametrize("precision,tol", [("3xtf32", 1e-3), ("fp32", 1e-3), ("tf32", 2e-2), ("bf16", 2e-2)])
def test_resnet18_graph(ob, r18_ref, precision, tol):
    nodes, inits, ins, outs, x, ref = r18_ref
    h = ob.Handle(0, precision=precision)
    g = ob.Graph(h, nodes, inits, ins, outs)
    st = g.stats()
    assert st["n_fused"] >= 20 + 8 + 17  # BN per conv, residual Adds, Relus
    xin = torch.from_numpy(x).cuda()
    y_eager = g.run([xin])[0].clone()
    y_graph = g.run([xin])[0].clone()  # captured
    y_replay = g.run([xin])[0]
    h.synchronize()
    np.testing.assert_array_equal(y_eager.cpu().numpy(), y_graph.cpu().numpy())
    np.testing.assert_array_equal(y_graph.cpu().numpy(), y_replay.cpu().numpy())
    check_logits(y_replay.cpu().numpy(), ref, tol, f"resnet18/{precision}")
    # host buffers in / out
    yh = g.run_host([x])[0]
    np.testing.assert_array_equal(yh, y_replay.cpu().numpy())
    # a pipelined sequence of host batches (each input copy overlaps the
    # previous batch's compute): every batch as if run alone
    xs = [x, (x * 0.5).astype(np.float32), x[::-1].copy()]
    pinned = [torch.from_numpy(v).pin_memory() for v in xs]
    outs = [[torch.empty(list(y_replay.shape), dtype=torch.float32).pin_memory()] for _ in xs]
    g.run_host_pipelined([[t] for t in pinned], outs)
    for v, o in zip(xs, outs):
        single = g.run([torch.from_numpy(v).cuda()])[0]
        h.synchronize()
        np.testing.assert_array_equal(o[0].numpy(), single.cpu().numpy())
    assert g.stats()["captured"] == 1
    g.close()
    h.close()


def test_graph_from_onnx_model(ob, r18_ref, tmp_path):
    """A .onnx file (weights in an external data file, symbolic batch
    dimension) read by onnxb200_model_load and built by
    onnxb200_graph_build_from_model runs exactly like the node-list graph."""
    nodes, inits, ins, outs, x, ref = r18_ref
    h = ob.Handle(0, precision="3xtf32")
    g_nodes = ob.Graph(h, nodes, inits, ins, outs)
    xin = torch.from_numpy(x).cuda()
    y_nodes = g_nodes.run([xin])[0].cpu().numpy()
    path = str(tmp_path / "resnet18.onnx")
    ob.onnx_io.save(path, nodes, inits, [("X", ["batch", 3, 224, 224])], outs, external_data=True)
    m = ob.onnx_io.load(path)
    assert m.inputs == [("X", [-1, 3, 224, 224])]
    with pytest.raises(ob.ValidationError):
        ob.Graph.from_model(h, m)  # symbolic batch and no shape given
    g = ob.Graph.from_model(h, m, {"X": list(x.shape)})
    assert g.output_shapes == g_nodes.output_shapes
    assert g.stats()["n_fused"] == g_nodes.stats()["n_fused"]
    y = g.run([xin])[0].cpu().numpy()
    np.testing.assert_array_equal(y, y_nodes)
    check_logits(y, ref, 1e-3, "resnet18 from .onnx")
    g.close()
    g_nodes.close()
    h.close()


def test_resnet18_full_batch_config(ob, oracle, r18_ref):
    """ResNet-18 at batch 32 (seed 2): images 0 and 31 against the oracle."""
    nodes, inits, ins, outs = ob.workloads.resnet18(batch=32, seed=2)
    x = ob.workloads.resnet_input(2, 32)
    h = ob.Handle(0, precision="3xtf32")
    g = ob.Graph(h, nodes, inits, ins, outs)
    y = g.run([torch.from_numpy(x).cuda()])[0]
    h.synchronize()
    y = y.cpu().numpy()
    n1, i1, _, _ = ob.workloads.resnet18(batch=1, seed=2)
    for i in (0, 31):
        ref = oracle.run_graph(n1, i1, {"X": x[i:i + 1]}, outs)[outs[0]]
        check_logits(y[i:i + 1], ref, 1e-3, f"resnet18 b32 image {i}")
    g.close()
    h.close()


def test_resnet50_full_batch_config(ob, oracle):
    """ResNet-50 v1.5 at batch 256 (seed 4), 3xTF32: images 0 and 255 against the oracle."""
    nodes, inits, ins, outs = ob.workloads.resnet50(batch=256, seed=4)
    x = ob.workloads.resnet_input(4, 256)
    h = ob.Handle(0, precision="3xtf32")
    g = ob.Graph(h, nodes, inits, ins, outs)
    st = g.stats()
    assert st["n_steps"] < len(nodes) / 2
    y = g.run([torch.from_numpy(x).cuda()])[0]
    h.synchronize()
    y = y.cpu().numpy()
    n1, i1, _, _ = ob.workloads.resnet50(batch=1, seed=4)
    for i in (0, 255):
        ref = oracle.run_graph(n1, i1, {"X": x[i:i + 1]}, outs)[outs[0]]
        check_logits(y[i:i + 1], ref, 1e-3, f"resnet50 b256 image {i}")
    g.close()
    h.close()


@pytest.mark.parametrize("precision", ["tf32", "bf16"])
def test_resnet50_fast_modes(ob, oracle, precision):
    nodes, inits, ins, outs = ob.workloads.resnet50(batch=2, seed=4)
    x = ob.workloads.resnet_input(4, 2)
    ref = oracle.run_graph(nodes, inits, {"X": x}, outs)[outs[0]]
    h = ob.Handle(0, precision=precision)
    g = ob.Graph(h, nodes, inits, ins, outs)
    y = g.run([torch.from_numpy(x).cuda()])[0]
    h.synchronize()
    check_logits(y.cpu().numpy(), ref, 2e-2, f"resnet50/{precision}")
    g.close()
    h.close()
