"""numpy/ctypes front end of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and
by the CPU-baseline leg of ``bench.py``, as the checker or as the timed CPU
baseline.  The product package never imports this module.

Every op takes and returns NCHW float32 numpy arrays, mirroring the reference's
``Operator::compute`` on ``Tensor { data: ArrayD<f32> }`` (src/ops/registry.rs:14-27,
src/ops/tensor.rs:206-218).  ``run_graph`` evaluates an ONNX-style node list with
these ops one node at a time, the way the reference's ExecutionEngine::run_node
would (src/execution/engine.rs:234-337), with no fusion.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i64 = ctypes.c_int64


class OracleError(RuntimeError):
    """Raised where the reference returns Err(Error::ValidationError/UnsupportedFeature)."""


def build(force: bool = False) -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    src = os.path.join(_HERE, "oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
    return _lib


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)


def _fp(a: Optional[np.ndarray]):
    if a is None:
        return ctypes.cast(None, _f32p)
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


def _shape_arr(shape: Sequence[int]):
    arr = (ctypes.c_int64 * max(1, len(shape)))(*[int(s) for s in shape])
    return arr


def _c32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _check(rc: int, what: str):
    if rc != 0:
        raise OracleError(f"{what}: oracle status {rc}")


# --------------------------------------------------------------------------- shapes
def conv_out_dim(inp, k, stride, pad_head, pad_tail, dilation) -> int:
    return int(lib().orc_conv_out_dim(_i64(inp), _i64(k), _i64(stride), _i64(pad_head),
                                      _i64(pad_tail), _i64(dilation)))


lib_restype_set = False


def _setup():
    global lib_restype_set
    if lib_restype_set:
        return
    L = lib()
    L.orc_conv_out_dim.restype = ctypes.c_int64
    L.orc_conv_strategy.restype = ctypes.c_int
    lib_restype_set = True


def same_pads(inp, k, stride, dilation, upper=True):
    _setup()
    h, t = ctypes.c_int64(), ctypes.c_int64()
    lib().orc_same_pads(_i64(inp), _i64(k), _i64(stride), _i64(dilation), 1 if upper else 2,
                        ctypes.byref(h), ctypes.byref(t))
    return int(h.value), int(t.value)


def conv_strategy(kh, kw, group) -> int:
    _setup()
    return int(lib().orc_conv_strategy(_i64(kh), _i64(kw), _i64(group)))


# --------------------------------------------------------------------------- ops
def conv2d(x, w, b=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1,
           auto_pad="NOTSET", strategy=0, acc64=False, nthreads=None) -> np.ndarray:
    """Conv::compute (conv.rs:156-203) for 2-D NCHW input."""
    _setup()
    x, w = _c32(x), _c32(w)
    b = None if b is None else _c32(b)
    n, c, h, wd = x.shape
    co, cg, kh, kw = w.shape
    if cg * group != c:
        raise OracleError("Conv: inconsistent channel dimensions")
    sh, sw = strides
    dh, dw = dilations
    if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
        up = auto_pad == "SAME_UPPER"
        pt, pb = same_pads(h, kh, sh, dh, up)
        pl, pr = same_pads(wd, kw, sw, dw, up)
    elif auto_pad == "VALID":
        pt = pl = pb = pr = 0
    else:
        pt, pl, pb, pr = pads
    oh = conv_out_dim(h, kh, sh, pt, pb, dh)
    ow = conv_out_dim(wd, kw, sw, pl, pr, dw)
    y = np.empty((n, co, oh, ow), np.float32)
    rc = lib().orc_conv2d(_fp(x), _i64(n), _i64(c), _i64(h), _i64(wd), _fp(w), _i64(co), _i64(kh),
                          _i64(kw), _fp(b), _i64(sh), _i64(sw), _i64(pt), _i64(pl), _i64(pb),
                          _i64(pr), _i64(dh), _i64(dw), _i64(group), ctypes.c_int(strategy),
                          ctypes.c_int(1 if acc64 else 0),
                          ctypes.c_int(nthreads or default_threads()), _fp(y))
    _check(rc, "Conv")
    return y


def conv_nd_direct(x, w, b=None, strides=None, pads=None, dilations=None, group=1):
    """compute_conv_direct (conv.rs:609-706) for 1-D, 2-D and 3-D inputs."""
    x, w = _c32(x), _c32(w)
    sd = x.ndim - 2
    strides = strides or [1] * sd
    dilations = dilations or [1] * sd
    pads = pads or [0] * (2 * sd)
    ys = (ctypes.c_int64 * 5)()
    out = [x.shape[0], w.shape[0]] + [
        conv_out_dim(x.shape[i + 2], w.shape[i + 2], strides[i], pads[i], pads[i + sd], dilations[i])
        for i in range(sd)]
    y = np.empty(out, np.float32)
    rc = lib().orc_conv_nd_direct(_fp(x), _shape_arr(x.shape), ctypes.c_int(x.ndim), _fp(w),
                                  _shape_arr(w.shape), _fp(None if b is None else _c32(b)),
                                  _shape_arr(strides), _shape_arr(pads), _shape_arr(dilations),
                                  _i64(group), _fp(y), ys)
    _check(rc, "Conv")
    return y


def matmul_shape(a_shape, b_shape) -> List[int]:
    out = (ctypes.c_int64 * 10)()
    ro = ctypes.c_int()
    rc = lib().orc_matmul_shape(_shape_arr(a_shape), ctypes.c_int(len(a_shape)), _shape_arr(b_shape),
                                ctypes.c_int(len(b_shape)), out, ctypes.byref(ro))
    _check(rc, "MatMul shape")
    return [int(out[i]) for i in range(ro.value)]


def matmul(a, b, acc64=False, nthreads=None) -> np.ndarray:
    """compute_matmul (matmul.rs:124-279)."""
    a, b = _c32(a), _c32(b)
    shape = matmul_shape(a.shape, b.shape)
    y = np.empty(shape, np.float32)
    rc = lib().orc_matmul(_fp(a), _shape_arr(a.shape), ctypes.c_int(a.ndim), _fp(b),
                          _shape_arr(b.shape), ctypes.c_int(b.ndim), ctypes.c_int(1 if acc64 else 0),
                          ctypes.c_int(nthreads or default_threads()), _fp(y))
    _check(rc, "MatMul")
    return y


def gemm(a, b, c=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0, acc64=False) -> np.ndarray:
    """ONNX Gemm; compute_gemm (gemm.rs:172-291) with attributes honoured."""
    a, b = _c32(a), _c32(b)
    m, k = (a.shape[1], a.shape[0]) if trans_a else a.shape
    k2, n = (b.shape[1], b.shape[0]) if trans_b else b.shape
    if k != k2:
        raise OracleError("Gemm: incompatible dimensions")
    cc = None if c is None else _c32(c)
    y = np.empty((m, n), np.float32)
    cs = _shape_arr(cc.shape if cc is not None else [1])
    rc = lib().orc_gemm(_fp(a), _fp(b), _fp(cc), cs, ctypes.c_int(0 if cc is None else cc.ndim),
                        _i64(m), _i64(n), _i64(k), ctypes.c_int(trans_a), ctypes.c_int(trans_b),
                        ctypes.c_float(alpha), ctypes.c_float(beta), ctypes.c_int(1 if acc64 else 0),
                        _fp(y))
    _check(rc, "Gemm")
    return y


def maxpool2d(x, kernel=(3, 3), strides=(2, 2), pads=(1, 1, 1, 1), ceil_mode=0,
              with_indices=False):
    """max_pool (pool.rs:307-393) called with explicit ONNX attributes."""
    x = _c32(x)
    n, c, h, w = x.shape
    kh, kw = kernel
    sh, sw = strides
    pt, pl, pb, pr = pads
    if ceil_mode:
        oh = (h + pt + pb - kh + sh - 1) // sh + 1
        ow = (w + pl + pr - kw + sw - 1) // sw + 1
    else:
        oh = (h + pt + pb - kh) // sh + 1
        ow = (w + pl + pr - kw) // sw + 1
    y = np.empty((n, c, oh, ow), np.float32)
    idx = np.empty((n, c, oh, ow), np.int64) if with_indices else None
    rc = lib().orc_maxpool2d(_fp(x), _i64(n), _i64(c), _i64(h), _i64(w), _i64(kh), _i64(kw),
                             _i64(sh), _i64(sw), _i64(pt), _i64(pl), _i64(pb), _i64(pr),
                             ctypes.c_int(ceil_mode), _fp(y),
                             idx.ctypes.data_as(_i64p) if idx is not None else ctypes.cast(None, _i64p))
    _check(rc, "MaxPool")
    return (y, idx) if with_indices else y


def global_avgpool(x) -> np.ndarray:
    """global_pool(GlobalAverage) (pool.rs:493-557)."""
    x = _c32(x)
    n, c = x.shape[:2]
    sp = int(np.prod(x.shape[2:])) if x.ndim > 2 else 1
    y = np.empty((n, c) + (1,) * (x.ndim - 2), np.float32)
    _check(lib().orc_global_avgpool(_fp(x), _i64(n), _i64(c), _i64(sp), _fp(y)), "GlobalAveragePool")
    return y


def relu(x) -> np.ndarray:
    """relu (activations.rs:244-246)."""
    x = _c32(x)
    y = np.empty_like(x)
    lib().orc_relu(_fp(x), _i64(x.size), _fp(y))
    return y


def broadcast_shape(a_shape, b_shape) -> List[int]:
    out = (ctypes.c_int64 * 16)()
    ro = ctypes.c_int()
    rc = lib().orc_broadcast_shape(_shape_arr(a_shape), ctypes.c_int(len(a_shape)), _shape_arr(b_shape),
                                   ctypes.c_int(len(b_shape)), out, ctypes.byref(ro))
    _check(rc, "broadcast")
    return [int(out[i]) for i in range(ro.value)]


def add(a, b) -> np.ndarray:
    """element_wise_binary_op(+) (tensor.rs:1124-1218)."""
    a, b = _c32(a), _c32(b)
    y = np.empty(broadcast_shape(a.shape, b.shape), np.float32)
    rc = lib().orc_add(_fp(a), _shape_arr(a.shape), ctypes.c_int(a.ndim), _fp(b), _shape_arr(b.shape),
                       ctypes.c_int(b.ndim), _fp(y))
    _check(rc, "Add")
    return y


def batchnorm(x, scale, bias, mean, var, eps=1e-5) -> np.ndarray:
    """ONNX BatchNormalization (inference); the reference has no such operator."""
    x = _c32(x)
    n, c = x.shape[:2]
    sp = int(np.prod(x.shape[2:])) if x.ndim > 2 else 1
    y = np.empty_like(x)
    rc = lib().orc_batchnorm(_fp(x), _i64(n), _i64(c), _i64(sp), _fp(_c32(scale)), _fp(_c32(bias)),
                             _fp(_c32(mean)), _fp(_c32(var)), ctypes.c_float(eps), _fp(y))
    _check(rc, "BatchNormalization")
    return y


# --------------------------------------------------------------------------- graphs
def run_graph(nodes: Sequence[dict], weights: Dict[str, np.ndarray], feeds: Dict[str, np.ndarray],
              outputs: Sequence[str], acc64=False, nthreads=None) -> Dict[str, np.ndarray]:
    """Evaluate an ONNX-style node list node by node with the oracle ops.

    Each node is ``{"op": str, "inputs": [names], "outputs": [names], "attrs": {...}}``.
    """
    env: Dict[str, np.ndarray] = dict(weights)
    env.update(feeds)
    for nd in nodes:
        op, ins, outs, at = nd["op"], nd["inputs"], nd["outputs"], nd.get("attrs", {})
        v = [env[i] if i else None for i in ins]
        if op == "Conv":
            y = conv2d(v[0], v[1], v[2] if len(v) > 2 else None, strides=at.get("strides", (1, 1)),
                       pads=at.get("pads", (0, 0, 0, 0)), dilations=at.get("dilations", (1, 1)),
                       group=at.get("group", 1), auto_pad=at.get("auto_pad", "NOTSET"),
                       acc64=acc64, nthreads=nthreads)
        elif op == "BatchNormalization":
            y = batchnorm(v[0], v[1], v[2], v[3], v[4], at.get("epsilon", 1e-5))
        elif op == "Relu":
            y = relu(v[0])
        elif op == "Add":
            y = add(v[0], v[1])
        elif op == "MaxPool":
            y = maxpool2d(v[0], at["kernel_shape"], at.get("strides", (1, 1)), at.get("pads", (0, 0, 0, 0)),
                          at.get("ceil_mode", 0))
        elif op == "GlobalAveragePool":
            y = global_avgpool(v[0])
        elif op == "Flatten":
            axis = at.get("axis", 1)
            y = v[0].reshape(int(np.prod(v[0].shape[:axis])), -1)
        elif op == "Gemm":
            y = gemm(v[0], v[1], v[2] if len(v) > 2 else None, at.get("alpha", 1.0), at.get("beta", 1.0),
                     at.get("transA", 0), at.get("transB", 0), acc64=acc64)
        elif op == "MatMul":
            y = matmul(v[0], v[1], acc64=acc64, nthreads=nthreads)
        else:
            raise OracleError(f"oracle: unsupported op {op}")
        env[outs[0]] = y
    return {o: env[o] for o in outputs}
