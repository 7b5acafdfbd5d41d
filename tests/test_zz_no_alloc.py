"""GPU test of onnxb200_conv2d_nhwc_noalloc, the convolution entry point for
callers that cannot call cudaMalloc while they run (a host framework that owns
all device memory and passes in pre-sized buffers, or a serving loop that must
not allocate).  It keeps its scratch -- packed weights and epilogue vectors --
in one fixed device array inside the library instead of a growable workspace.

Checked here through the C ABI: two calls in a row (different inputs, weights
and epilogues) each match the regular entry point onnxb200_conv2d within the
3xTF32 tolerance used by the other tests (rtol 1e-5 / atol 1e-4); device free
memory does not change across those calls; oversize and NCHW requests are
refused with status codes.  This file is collected last so that a run that
stops at the first failure has already run every other test.
"""
import ctypes
import importlib

import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu

C = importlib.import_module("onnx-rs_b200")._capi


def desc_nhwc(x_shape, w_shape, pad, stride, epilogue):
    d = C.ConvDesc()
    d.n, d.h, d.w, d.c = x_shape
    d.c_out, _, d.kh, d.kw = w_shape
    d.stride_h = d.stride_w = stride
    d.pad_top = d.pad_left = d.pad_bottom = d.pad_right = pad
    d.dil_h = d.dil_w = 1
    d.group = 1
    d.layout = C.LAYOUT_NHWC
    d.epilogue = epilogue
    d.precision = C.PREC_3XTF32
    d.bn_epsilon = 1e-5
    return d


def p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def make_case(seed, n, c, hw, co, k, stride, with_bn, with_res):
    rng = np.random.default_rng(seed)
    pad = k // 2
    x = torch.from_numpy(rng.standard_normal((n, hw, hw, c)).astype(np.float32)).cuda()
    w = torch.from_numpy((rng.standard_normal((co, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.uniform(-0.1, 0.1, co).astype(np.float32)).cuda()
    bn = None
    if with_bn:
        bn = [torch.from_numpy(v.astype(np.float32)).cuda() for v in
              (rng.uniform(0.5, 1.5, co), rng.uniform(-0.2, 0.2, co), rng.normal(0, 0.1, co), rng.uniform(0.5, 1.5, co))]
    oh = (hw + 2 * pad - k) // stride + 1
    res = torch.from_numpy(rng.standard_normal((n, oh, oh, co)).astype(np.float32)).cuda() if with_res else None
    epi = C.EPI_BIAS | C.EPI_RELU | (C.EPI_BN if with_bn else 0) | (C.EPI_RESIDUAL if with_res else 0)
    d = desc_nhwc((n, hw, hw, c), (co, c, k, k), pad, stride, epi)
    return d, x, w, b, bn, res, (n, oh, oh, co)


def run_regular(handle, d, x, w, b, bn, res, out_shape):
    y = torch.empty(out_shape, dtype=torch.float32, device="cuda")
    bnp = bn or [None] * 4
    handle.check(C.lib().onnxb200_conv2d(handle.ptr, ctypes.byref(d), p(x), p(w), p(b), p(bnp[0]), p(bnp[1]),
                                         p(bnp[2]), p(bnp[3]), p(res), p(y)), "conv2d")
    handle.synchronize()
    return y


def run_noalloc(d, x, w, b, bn, res, out_shape, y=None):
    if y is None:
        y = torch.empty(out_shape, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    bnp = bn or [None] * 4
    rc = C.lib().onnxb200_conv2d_nhwc_noalloc(None, ctypes.byref(d), p(x), p(w), p(b), p(bnp[0]), p(bnp[1]),
                                               p(bnp[2]), p(bnp[3]), p(res), p(y))
    return rc, y


def test_noalloc_matches_regular_entry_twice(handle):
    cases = [make_case(1, 8, 256, 14, 256, 3, 1, with_bn=True, with_res=True),
             make_case(2, 4, 64, 28, 128, 3, 2, with_bn=False, with_res=False)]
    # first call on this device does the one-time symbol lookup
    rc, _ = run_noalloc(*cases[1])
    assert rc == 0
    outs = [torch.empty(case[6], dtype=torch.float32, device="cuda") for case in cases]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for case, y in zip(cases, outs):  # two calls in a row through the C ABI
        rc, _ = run_noalloc(*case, y=y)
        assert rc == 0, C.lib().onnxb200_status_string(rc)
    torch.cuda.synchronize()
    # the calls themselves allocated nothing (outputs were allocated before)
    assert torch.cuda.mem_get_info()[0] == free_before
    for case, y in zip(cases, outs):
        ref = run_regular(handle, *case)
        assert_close(y.cpu().numpy(), ref.cpu().numpy(), 1e-5, 1e-4, "noalloc vs onnxb200_conv2d")


def test_noalloc_rejects_what_it_cannot_hold():
    # 1024 x (3*3*1024) packed hi+lo weights = 75 MB > the fixed array
    d, x, w, b, bn, res, shape = make_case(3, 1, 1024, 7, 1024, 3, 1, with_bn=False, with_res=False)
    rc, _ = run_noalloc(d, x, w, b, bn, res, shape)
    assert rc == C.ERR_RESOURCE_EXHAUSTED
    d2, x, w, b, bn, res, shape = make_case(4, 1, 16, 8, 16, 3, 1, with_bn=False, with_res=False)
    d2.layout = C.LAYOUT_NCHW
    rc, _ = run_noalloc(d2, x, w, b, bn, res, shape)
    assert rc == C.ERR_VALIDATION


def test_noalloc_refuses_a_capturing_stream():
    """The entry point blocks until y is written, which a stream under capture
    cannot do: it returns ERR_UNSUPPORTED there and leaves the capture intact."""
    d, x, w, b, bn, res, shape = make_case(5, 1, 16, 8, 16, 3, 1, with_bn=False, with_res=False)
    y = torch.zeros(shape, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = C.lib().onnxb200_conv2d_nhwc_noalloc(s, ctypes.byref(d), p(x), p(w), p(b), None, None, None, None,
                                                   None, p(y))
        y.add_(1.0)
    assert rc == C.ERR_UNSUPPORTED
    graph.replay()
    torch.cuda.synchronize()
    assert float(y.min()) == 1.0 and float(y.max()) == 1.0
