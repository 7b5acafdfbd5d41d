"""Host-side mirror of the reference's operator interface on top of the C ABI.

``Operator`` follows ``trait Operator`` (src/ops/registry.rs:14-27): ``compute``
takes input tensors and returns freshly allocated outputs (the reference replaces
``outputs[i]`` wholesale, src/ops/nn/conv.rs:199-200), ``output_shapes`` infers
shapes from a node, ``validate`` checks a node.  Tensors are NCHW fp32 torch CUDA
tensors.  Unlike the reference's ``compute`` (which ignores node attributes,
src/ops/nn/conv.rs:180-199, src/ops/math/gemm.rs:35-38), operators built with
``from_node`` carry the node's attributes.

``OperatorRegistry`` keeps the reference's (name, domain, version) keys
(src/ops/registry.rs:30-98); ``create_operator_for_node`` resolves the newest
registered version not above the requested opset (the reference compares
character codes instead, src/ops/registry.rs:105-106, and never matches).
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence

import torch

from . import _capi as C
from .runtime import (Handle, InvalidOperator, UnsupportedFeature, ValidationError, dptr)


class ExecutionContext:
    """Operator-level context (src/ops/registry.rs:8-11) plus the device handle."""

    def __init__(self, handle: Handle, options: Optional[Dict[str, str]] = None):
        self.handle = handle
        self.options = dict(options or {})


def _attrs(node) -> dict:
    return dict(node.get("attrs", {})) if isinstance(node, dict) else dict(getattr(node, "attrs", {}))


def _prec(ctx: ExecutionContext, prec) -> int:
    if prec is None:
        p = ctx.options.get("precision")
        return C.PRECISIONS[p] if p else C.PREC_DEFAULT
    return C.PRECISIONS[prec] if isinstance(prec, str) else int(prec)


class Operator:
    op_type = ""

    def compute(self, inputs: Sequence[Optional[torch.Tensor]], ctx: ExecutionContext) -> List[torch.Tensor]:
        raise NotImplementedError

    def input_shapes(self, node, input_shapes):
        return list(input_shapes)

    def output_shapes(self, node, input_shapes) -> List[Optional[List[int]]]:
        raise NotImplementedError

    def validate(self, node) -> None:
        n_in = len(node["inputs"]) if isinstance(node, dict) else len(node.inputs)
        if n_in < self.min_inputs:
            raise ValidationError(C.ERR_VALIDATION,
                                  f"{self.op_type} operator requires at least {self.min_inputs} inputs, got {n_in}")

    min_inputs = 1


# --------------------------------------------------------------------------- Conv
class Conv(Operator):
    """Conv (src/ops/nn/conv.rs:115-323): 2-D with an optional fused epilogue
    (BatchNormalization, residual Add, Relu) on the tensor-core path; 1-D (NCL,
    run as 2-D of height 1) and 3-D (NCDHW, CUDA cores) with bias and Relu.
    strides / pads / dilations default per rank (ONNX: ones, zeros, ones)."""
    op_type = "Conv"
    min_inputs = 2

    def __init__(self, strides=None, pads=None, dilations=None, group=1, auto_pad="NOTSET",
                 precision=None, relu=False):
        self.strides = None if strides is None else list(strides)
        self.pads = None if pads is None else list(pads)
        self.dilations = None if dilations is None else list(dilations)
        self.group = int(group)
        self.auto_pad = auto_pad
        self.precision = precision
        self.relu = relu

    @classmethod
    def from_node(cls, node, **kw):
        a = _attrs(node)
        return cls(a.get("strides"), a.get("pads"), a.get("dilations"), a.get("group", 1),
                   a.get("auto_pad", "NOTSET"), **kw)

    def _attr(self, sp):
        """strides, pads (begin..., end...), dilations for `sp` spatial dims."""
        st = self.strides if self.strides is not None else [1] * sp
        pd = self.pads if self.pads is not None else [0] * (2 * sp)
        dl = self.dilations if self.dilations is not None else [1] * sp
        if len(st) != sp or len(pd) != 2 * sp or len(dl) != sp:
            raise ValidationError(C.ERR_VALIDATION, f"Conv: attributes do not match {sp} spatial dims")
        return st, pd, dl

    def nd_desc(self, x_shape, w_shape):
        """onnxb200_conv_nd_desc for a 1-D, 2-D or 3-D input."""
        sp = len(x_shape) - 2
        if sp < 1 or sp > 3 or len(w_shape) != len(x_shape):
            raise ValidationError(C.ERR_VALIDATION, "Conv supports only 1D, 2D, and 3D convolutions")
        st, pd, dl = self._attr(sp)
        d = C.ConvNdDesc()
        d.spatial = sp
        d.n, d.c = x_shape[0], x_shape[1]
        d.c_out = w_shape[0]
        d.group = self.group
        for i in range(sp):
            d.in_[i] = x_shape[2 + i]
            d.kernel[i] = w_shape[2 + i]
            d.stride[i] = st[i]
            d.pad_begin[i] = pd[i]
            d.pad_end[i] = pd[sp + i]
            d.dilation[i] = dl[i]
        d.auto_pad = C.AUTOPAD[self.auto_pad]
        d.relu = 1 if self.relu else 0
        return d

    def desc(self, x_shape, w_shape, layout=C.LAYOUT_NCHW, epilogue=0, prec=C.PREC_DEFAULT, eps=1e-5):
        d = C.ConvDesc()
        if layout == C.LAYOUT_NHWC:
            d.n, d.h, d.w, d.c = x_shape
        else:
            d.n, d.c, d.h, d.w = x_shape
        d.c_out, _, d.kh, d.kw = w_shape
        st, pd, dl = self._attr(2)
        d.stride_h, d.stride_w = st
        d.pad_top, d.pad_left, d.pad_bottom, d.pad_right = pd
        d.dil_h, d.dil_w = dl
        d.group = self.group
        d.auto_pad = C.AUTOPAD[self.auto_pad]
        d.layout = layout
        d.epilogue = epilogue
        d.precision = prec
        d.bn_epsilon = eps
        return d

    def output_shape(self, x_shape, w_shape) -> List[int]:
        if len(x_shape) != 4:
            d = self.nd_desc(x_shape, w_shape)
            out = C.i64_array([0] * 5)
            rank = ctypes.c_int()
            rc = C.lib().onnxb200_conv_nd_output_shape(ctypes.byref(d), out, ctypes.byref(rank))
            if rc != 0:
                raise ValidationError(rc, "Conv: invalid shapes or attributes")
            return [int(v) for v in out[:rank.value]]
        d = self.desc(x_shape, w_shape)
        out = C.i64_array([0] * 4)
        rc = C.lib().onnxb200_conv2d_output_shape(ctypes.byref(d), out)
        if rc != 0:
            raise ValidationError(rc, "Conv: invalid shapes or attributes")
        return [int(v) for v in out[:4]]

    def output_shapes(self, node, input_shapes):
        if len(input_shapes) < 2:
            raise ValidationError(C.ERR_VALIDATION, f"Conv requires at least 2 inputs, got {len(input_shapes)}")
        x, w = input_shapes[0], input_shapes[1]
        if x is None or w is None:
            return [None]
        return [type(self).from_node(node).output_shape(x, w)]

    def compute(self, inputs, ctx, bn=None, residual=None, layout=C.LAYOUT_NCHW):
        """inputs = [X, W, B?]; bn = (scale, B, mean, var, eps) fuses BatchNormalization."""
        x, w = inputs[0], inputs[1]
        b = inputs[2] if len(inputs) > 2 else None
        h = ctx.handle
        if x.dim() != 4:  # 1-D / 3-D: bias and Relu only
            if bn is not None or residual is not None or layout != C.LAYOUT_NCHW:
                raise UnsupportedFeature(C.ERR_UNSUPPORTED, "Conv: fused BN / residual / NHWC are 2-D only")
            y = torch.empty(self.output_shape(tuple(x.shape), tuple(w.shape)), dtype=torch.float32,
                            device=x.device)
            d = self.nd_desc(tuple(x.shape), tuple(w.shape))
            h.check(C.lib().onnxb200_conv_nd(h.ptr, ctypes.byref(d), dptr(x), dptr(w), dptr(b), dptr(y)), "Conv")
            return [y]
        epi = (C.EPI_BIAS if b is not None else 0) | (C.EPI_BN if bn is not None else 0) | \
              (C.EPI_RESIDUAL if residual is not None else 0) | (C.EPI_RELU if self.relu else 0)
        eps = bn[4] if bn is not None else 1e-5
        d = self.desc(tuple(x.shape), tuple(w.shape), layout, epi, _prec(ctx, self.precision), eps)
        out = C.i64_array([0] * 4)
        h.check(C.lib().onnxb200_conv2d_output_shape(ctypes.byref(d), out), "Conv")
        n, co, oh, ow = [int(v) for v in out[:4]]
        shape = (n, co, oh, ow) if layout == C.LAYOUT_NCHW else (n, oh, ow, co)
        y = torch.empty(shape, dtype=torch.float32, device=x.device)
        bnp = list(bn[:4]) if bn is not None else [None] * 4
        h.check(C.lib().onnxb200_conv2d(h.ptr, ctypes.byref(d), dptr(x), dptr(w), dptr(b), dptr(bnp[0]),
                                        dptr(bnp[1]), dptr(bnp[2]), dptr(bnp[3]), dptr(residual), dptr(y)), "Conv")
        return [y]


class ConvPlan:
    """Prepared convolution (onnxb200_conv_plan_*): weights packed and BN folded once.

    ``layout`` is the layout of x / residual / y at run time (NHWC runs the
    kernel directly on the caller's buffers)."""

    def __init__(self, ctx: ExecutionContext, conv: Conv, x_shape, w, bias=None, bn=None,
                 layout=C.LAYOUT_NHWC, residual=False):
        self.ctx = ctx
        h = ctx.handle
        epi = (C.EPI_BIAS if bias is not None else 0) | (C.EPI_BN if bn is not None else 0) | \
              (C.EPI_RESIDUAL if residual else 0) | (C.EPI_RELU if conv.relu else 0)
        self.desc = conv.desc(tuple(x_shape), tuple(w.shape), layout, epi, _prec(ctx, conv.precision),
                              bn[4] if bn is not None else 1e-5)
        out = C.i64_array([0] * 4)
        h.check(C.lib().onnxb200_conv2d_output_shape(ctypes.byref(self.desc), out), "Conv")
        n, co, oh, ow = [int(v) for v in out[:4]]
        self.out_shape = (n, co, oh, ow) if layout == C.LAYOUT_NCHW else (n, oh, ow, co)
        bnp = list(bn[:4]) if bn is not None else [None] * 4
        ptr = ctypes.c_void_p()
        h.check(C.lib().onnxb200_conv_plan_create(h.ptr, ctypes.byref(self.desc), dptr(w), dptr(bias),
                                                  dptr(bnp[0]), dptr(bnp[1]), dptr(bnp[2]), dptr(bnp[3]),
                                                  ctypes.byref(ptr)), "conv plan")
        self.ptr = ptr

    def run(self, x: torch.Tensor, y: torch.Tensor, residual: Optional[torch.Tensor] = None):
        h = self.ctx.handle
        h.check(C.lib().onnxb200_conv_plan_run(h.ptr, self.ptr, dptr(x), dptr(residual), dptr(y)), "conv plan run")
        return y

    def close(self):
        if getattr(self, "ptr", None):
            C.lib().onnxb200_conv_plan_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------- MatMul / Gemm
class MatMul(Operator):
    """MatMul (src/ops/math/matmul.rs:60-124): numpy-broadcast batched matmul."""
    op_type = "MatMul"
    min_inputs = 2

    def __init__(self, precision=None):
        self.precision = precision

    @classmethod
    def from_node(cls, node, **kw):
        return cls(**kw)

    @staticmethod
    def output_shape(a_shape, b_shape) -> List[int]:
        out = C.i64_array([0] * 10)
        r = ctypes.c_int()
        rc = C.lib().onnxb200_matmul_output_shape(C.i64_array(a_shape), len(a_shape), C.i64_array(b_shape),
                                                  len(b_shape), out, ctypes.byref(r))
        if rc != 0:
            raise ValidationError(rc, f"Incompatible shapes for MatMul: {list(a_shape)} and {list(b_shape)}")
        return [int(v) for v in out[:r.value]]

    def output_shapes(self, node, input_shapes):
        a, b = input_shapes[0], input_shapes[1]
        return [None if a is None or b is None else self.output_shape(a, b)]

    def compute(self, inputs, ctx, bias=None, relu=False):
        a, b = inputs[0], inputs[1]
        shape = self.output_shape(tuple(a.shape), tuple(b.shape))
        y = torch.empty(shape, dtype=torch.float32, device=a.device)
        h = ctx.handle
        h.check(C.lib().onnxb200_matmul(h.ptr, dptr(a), C.i64_array(a.shape), a.dim(), dptr(b),
                                        C.i64_array(b.shape), b.dim(), dptr(bias), C.EPI_RELU if relu else 0,
                                        _prec(ctx, self.precision), dptr(y)), "MatMul")
        return [y]


class Gemm(Operator):
    """Gemm (src/ops/math/gemm.rs:17-44) with alpha, beta, transA, transB honoured."""
    op_type = "Gemm"
    min_inputs = 2

    def __init__(self, alpha=1.0, beta=1.0, trans_a=0, trans_b=0, precision=None, relu=False):
        self.alpha, self.beta = float(alpha), float(beta)
        self.trans_a, self.trans_b = int(trans_a), int(trans_b)
        self.precision = precision
        self.relu = relu

    @classmethod
    def from_node(cls, node, **kw):
        a = _attrs(node)
        return cls(a.get("alpha", 1.0), a.get("beta", 1.0), a.get("transA", 0), a.get("transB", 0), **kw)

    def output_shapes(self, node, input_shapes):
        a, b = input_shapes[0], input_shapes[1]
        if a is None or b is None:
            return [None]
        g = type(self).from_node(node)
        m = a[1] if g.trans_a else a[0]
        n = b[0] if g.trans_b else b[1]
        return [[m, n]]

    def compute(self, inputs, ctx):
        a, b = inputs[0], inputs[1]
        c = inputs[2] if len(inputs) > 2 else None
        if a.dim() != 2 or b.dim() != 2:
            raise ValidationError(C.ERR_VALIDATION, "Gemm inputs must be 2D matrices")
        m, k = (a.shape[1], a.shape[0]) if self.trans_a else (a.shape[0], a.shape[1])
        k2, n = (b.shape[1], b.shape[0]) if self.trans_b else (b.shape[0], b.shape[1])
        if k != k2:
            raise ValidationError(C.ERR_VALIDATION, f"Incompatible dimensions for Gemm: {k} and {k2}")
        y = torch.empty((m, n), dtype=torch.float32, device=a.device)
        h = ctx.handle
        cs = C.i64_array(c.shape if c is not None else [1])
        h.check(C.lib().onnxb200_gemm(h.ptr, dptr(a), dptr(b), dptr(c), cs, 0 if c is None else c.dim(), m, n, k,
                                      self.trans_a, self.trans_b, self.alpha, self.beta,
                                      C.EPI_RELU if self.relu else 0, _prec(ctx, self.precision), dptr(y)), "Gemm")
        return [y]


# --------------------------------------------------------------------------- pooling
class MaxPool(Operator):
    """MaxPool (src/ops/nn/pool.rs:168-193) with the node's attributes (the
    reference hard-codes 2x2/2, pool.rs:185-187)."""
    op_type = "MaxPool"

    def __init__(self, kernel_shape=(2, 2), strides=(2, 2), pads=(0, 0, 0, 0), ceil_mode=0):
        self.kernel_shape, self.strides, self.pads = list(kernel_shape), list(strides), list(pads)
        self.ceil_mode = int(ceil_mode)

    @classmethod
    def from_node(cls, node, **kw):
        a = _attrs(node)
        return cls(a.get("kernel_shape", (2, 2)), a.get("strides", (1, 1)), a.get("pads", (0, 0, 0, 0)),
                   a.get("ceil_mode", 0))

    def out_hw(self, h, w):
        kh, kw = self.kernel_shape
        sh, sw = self.strides
        pt, pl, pb, pr = self.pads
        if self.ceil_mode:
            return (h + pt + pb - kh + sh - 1) // sh + 1, (w + pl + pr - kw + sw - 1) // sw + 1
        return (h + pt + pb - kh) // sh + 1, (w + pl + pr - kw) // sw + 1

    def output_shapes(self, node, input_shapes):
        x = input_shapes[0]
        if x is None:
            return [None]
        oh, ow = type(self).from_node(node).out_hw(x[2], x[3])
        return [[x[0], x[1], oh, ow]]

    def compute(self, inputs, ctx, with_indices=False, layout=C.LAYOUT_NCHW):
        x = inputs[0]
        if layout == C.LAYOUT_NHWC:
            n, hh, ww, c = x.shape
        else:
            n, c, hh, ww = x.shape
        oh, ow = self.out_hw(hh, ww)
        shape = (n, c, oh, ow) if layout == C.LAYOUT_NCHW else (n, oh, ow, c)
        y = torch.empty(shape, dtype=torch.float32, device=x.device)
        ind = torch.empty((n, c, oh, ow), dtype=torch.int64, device=x.device) if with_indices else None
        h = ctx.handle
        out = C.i64_array([0] * 4)
        h.check(C.lib().onnxb200_maxpool2d(h.ptr, layout, n, c, hh, ww, *self.kernel_shape, *self.strides,
                                           *self.pads, self.ceil_mode, dptr(x), dptr(y),
                                           None if ind is None else ctypes.c_void_p(ind.data_ptr()), out),
                "MaxPool")
        return [y, ind] if with_indices else [y]


class GlobalAveragePool(Operator):
    """GlobalAveragePool (src/ops/nn/pool.rs:275-295 -> global_pool :493-557)."""
    op_type = "GlobalAveragePool"

    @classmethod
    def from_node(cls, node, **kw):
        return cls()

    def output_shapes(self, node, input_shapes):
        x = input_shapes[0]
        return [None if x is None else [x[0], x[1]] + [1] * (len(x) - 2)]

    def compute(self, inputs, ctx, layout=C.LAYOUT_NCHW):
        x = inputs[0]
        if layout == C.LAYOUT_NHWC:
            n, hh, ww, c = x.shape
        else:
            n, c, hh, ww = x.shape
        y = torch.empty((n, c, 1, 1), dtype=torch.float32, device=x.device)
        h = ctx.handle
        h.check(C.lib().onnxb200_global_avgpool(h.ptr, layout, n, c, hh, ww, dptr(x), dptr(y)), "GlobalAveragePool")
        return [y]


# --------------------------------------------------------------------------- elementwise
class Relu(Operator):
    """Relu (src/ops/activations.rs:92-96, relu :244-246)."""
    op_type = "Relu"

    @classmethod
    def from_node(cls, node, **kw):
        return cls()

    def output_shapes(self, node, input_shapes):
        return [input_shapes[0]]

    def compute(self, inputs, ctx):
        x = inputs[0]
        y = torch.empty_like(x)
        ctx.handle.check(C.lib().onnxb200_relu(ctx.handle.ptr, dptr(x), x.numel(), dptr(y)), "Relu")
        return [y]


class Add(Operator):
    """Add = element_wise_binary_op(+) with broadcasting (src/ops/tensor.rs:1124-1218)."""
    op_type = "Add"
    min_inputs = 2

    def __init__(self, relu=False):
        self.relu = relu

    @classmethod
    def from_node(cls, node, **kw):
        return cls(**kw)

    @staticmethod
    def broadcast(a, b):
        r = max(len(a), len(b))
        a = [1] * (r - len(a)) + list(a)
        b = [1] * (r - len(b)) + list(b)
        out = []
        for i, (x, y) in enumerate(zip(a, b)):
            if x != y and x != 1 and y != 1:
                raise ValidationError(C.ERR_VALIDATION,
                                      f"Cannot broadcast shapes {a} and {b}: incompatible dimensions at index {i}")
            out.append(y if x == 1 else x)
        return out

    def output_shapes(self, node, input_shapes):
        a, b = input_shapes[0], input_shapes[1]
        return [None if a is None or b is None else self.broadcast(a, b)]

    def compute(self, inputs, ctx):
        a, b = inputs[0], inputs[1]
        y = torch.empty(self.broadcast(a.shape, b.shape), dtype=torch.float32, device=a.device)
        h = ctx.handle
        h.check(C.lib().onnxb200_add(h.ptr, dptr(a), C.i64_array(a.shape), a.dim(), dptr(b), C.i64_array(b.shape),
                                     b.dim(), 1 if self.relu else 0, dptr(y)), "Add")
        return [y]


class BatchNormalization(Operator):
    """ONNX BatchNormalization (inference).  Not in the reference registry."""
    op_type = "BatchNormalization"
    min_inputs = 5

    def __init__(self, epsilon=1e-5):
        self.epsilon = float(epsilon)

    @classmethod
    def from_node(cls, node, **kw):
        return cls(_attrs(node).get("epsilon", 1e-5))

    def output_shapes(self, node, input_shapes):
        return [input_shapes[0]]

    def compute(self, inputs, ctx, layout=C.LAYOUT_NCHW):
        x, scale, bias, mean, var = inputs[:5]
        if layout == C.LAYOUT_NHWC:
            n, hh, ww, c = x.shape
        else:
            n, c, hh, ww = x.shape
        y = torch.empty_like(x)
        h = ctx.handle
        h.check(C.lib().onnxb200_batchnorm(h.ptr, layout, n, c, hh, ww, dptr(x), dptr(scale), dptr(bias),
                                           dptr(mean), dptr(var), self.epsilon, dptr(y)), "BatchNormalization")
        return [y]


class Flatten(Operator):
    """ONNX Flatten (a view; the reference only infers its shape, src/memory/planner.rs:1735)."""
    op_type = "Flatten"

    def __init__(self, axis=1):
        self.axis = int(axis)

    @classmethod
    def from_node(cls, node, **kw):
        return cls(_attrs(node).get("axis", 1))

    def output_shapes(self, node, input_shapes):
        x = input_shapes[0]
        if x is None:
            return [None]
        ax = type(self).from_node(node).axis
        ax = ax + len(x) if ax < 0 else ax
        a = 1
        for v in x[:ax]:
            a *= v
        b = 1
        for v in x[ax:]:
            b *= v
        return [[a, b]]

    def compute(self, inputs, ctx):
        x = inputs[0]
        return [x.reshape(self.output_shapes({"attrs": {"axis": self.axis}}, [list(x.shape)])[0])]


# --------------------------------------------------------------------------- registry
class OperatorRegistry:
    """(name, domain, version)-keyed registry (src/ops/registry.rs:30-128)."""

    def __init__(self):
        self.operators: Dict[tuple, type] = {}

    def register_operator(self, name: str, domain: str, version: int, op_cls) -> None:
        key = (name, domain, int(version))
        if key in self.operators:
            raise InvalidOperator(C.ERR_INVALID_OPERATOR,
                                  f"Operator {domain}.{name} (version {version}) is already registered")
        self.operators[key] = op_cls

    def get_operator(self, name: str, domain: str, version: int):
        return self.operators.get((name, domain, int(version)))

    @classmethod
    def initialize_standard_operators(cls) -> "OperatorRegistry":
        r = cls()
        # versions as registered by the reference (src/ops/registry.rs:74-95); BN, Add
        # and Flatten are additions for this path.
        for name, ver, op in (("MatMul", 9, MatMul), ("Gemm", 9, Gemm), ("Conv", 11, Conv),
                              ("MaxPool", 11, MaxPool), ("GlobalAveragePool", 1, GlobalAveragePool),
                              ("Relu", 6, Relu), ("Add", 7, Add), ("BatchNormalization", 9, BatchNormalization),
                              ("Flatten", 9, Flatten)):
            r.register_operator(name, "", ver, op)
        return r

    def create_operator_for_node(self, node, opset: int = 17, **kw) -> Operator:
        name = node["op"] if isinstance(node, dict) else node.op_type
        domain = (node.get("domain", "") if isinstance(node, dict) else getattr(node, "domain", "")) or ""
        best = None
        for (n, d, v), op in self.operators.items():
            if n == name and d == domain and v <= opset and (best is None or v > best[0]):
                best = (v, op)
        if best is None:
            raise InvalidOperator(C.ERR_INVALID_OPERATOR,
                                  f"Operator {domain}.{name} (opset {opset}) not found in registry")
        return best[1].from_node(node, **kw)
