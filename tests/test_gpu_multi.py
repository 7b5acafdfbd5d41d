"""Batch-sharded replicas on several GPUs of one process (onnxb200_multi_*):
the concatenated logits of all devices against the oracle on the full batch,
and each device's rows bit-identical to a one-device graph of that slice."""
import importlib

import numpy as np
import pytest
import torch

from test_gpu_graph import check_logits_3x, oracle_logits

pytestmark = pytest.mark.gpu

ob_mod = importlib.import_module("onnx-rs_b200")


def test_multi_one_device_matches_graph(ob):
    nodes, inits, ins, outs = ob.workloads.resnet18(batch=8, seed=2)
    x = ob.workloads.resnet_input(2, 8)
    m = ob.MultiGraph([0], nodes, inits, ins, outs)
    assert m.output_shapes == [[8, 1000]]
    y = m.run_host([[x], [x * 0.5]])
    h = ob.Handle(0, precision="3xtf32")
    g = ob.Graph(h, nodes, inits, ins, outs)
    np.testing.assert_array_equal(y[0][0], g.run_host([x])[0])
    np.testing.assert_array_equal(y[1][0], g.run_host([(x * 0.5).astype(np.float32)])[0])
    info = m.info()
    assert info["n_devices"] == 1 and info["batch"] == 8 and info["slice_begin"] == [0]
    assert info["last_run_ms"][0] > 0
    g.close()
    h.close()
    m.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multi_two_devices_resnet50(ob, oracle):
    """ResNet-50 v1.5 (seed 4), 32 images split 16 + 16 over two GPUs: all 32
    logit rows against the oracle on the full batch; device 1's rows equal a
    one-device graph of the same 16 images."""
    nodes, inits, ins, outs = ob.workloads.resnet50(batch=32, seed=4)
    x = ob.workloads.resnet_input(4, 32)
    m = ob.MultiGraph([0, 1], nodes, inits, ins, outs)
    hx = torch.from_numpy(x).pin_memory()
    hy = torch.empty((32, 1000), dtype=torch.float32).pin_memory()
    m.run_host([[hx]], [[hy]])
    y = hy.numpy().copy()
    info = m.info()
    assert info["slice_begin"] == [0, 16] and all(t > 0 for t in info["last_run_ms"])
    m.close()
    r32 = oracle_logits(oracle, nodes, inits, x, outs, np.arange(32), False)
    r64 = oracle_logits(oracle, nodes, inits, x, outs, np.arange(32), True)
    check_logits_3x(y, r32, r64, "resnet50 b32 over 2 GPUs")
    n16, i16, ins16, _ = ob.workloads.resnet50(batch=16, seed=4)
    h = ob.Handle(0, precision="3xtf32")
    g = ob.Graph(h, n16, i16, ins16, outs)
    np.testing.assert_array_equal(y[16:], g.run_host([x[16:]])[0])
    g.close()
    h.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multi_uneven_slices(ob):
    """33 images over two devices: 17 + 16, rows land in the right places."""
    nodes, inits, ins, outs = ob.workloads.resnet18(batch=33, seed=2)
    x = ob.workloads.resnet_input(2, 33)
    m = ob.MultiGraph([0, 1], nodes, inits, ins, outs)
    y = m.run_host([[x]])[0][0]
    assert m.info()["slice_begin"] == [0, 17]
    m.close()
    for lo, hi in ((0, 17), (17, 33)):
        nb, ib, insb, _ = ob.workloads.resnet18(batch=hi - lo, seed=2)
        h = ob.Handle(0, precision="3xtf32")
        g = ob.Graph(h, nb, ib, insb, outs)
        np.testing.assert_array_equal(y[lo:hi], g.run_host([x[lo:hi]])[0])
        g.close()
        h.close()
