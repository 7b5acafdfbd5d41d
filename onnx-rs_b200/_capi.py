"""ctypes binding of libonnxb200.so (the C ABI declared in include/onnxb200.h).

The library must be built in-tree (``make -C onnx-rs_b200/csrc``); importing a
compute entry point without it raises immediately -- there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libonnxb200.so")

# status codes (include/onnxb200.h)
OK = 0
ERR_VALIDATION = 1
ERR_EXECUTION = 2
ERR_UNSUPPORTED = 3
ERR_TIMEOUT = 4
ERR_RESOURCE_EXHAUSTED = 5
ERR_INVALID_GRAPH = 6
ERR_INVALID_OPERATOR = 7
ERR_CANCELLED = 8
ERR_INVALID_ARGUMENT = 9
ERR_IO = 10
ERR_PROTOBUF = 11
ERR_INVALID_MODEL = 12

PREC_DEFAULT = -1
PREC_3XTF32 = 0
PREC_TF32 = 1
PREC_BF16 = 2
PREC_FP32 = 3
PRECISIONS = {"3xtf32": PREC_3XTF32, "tf32": PREC_TF32, "bf16": PREC_BF16, "fp32": PREC_FP32}

LAYOUT_NCHW = 0
LAYOUT_NHWC = 1

AUTOPAD = {"NOTSET": 0, "SAME_UPPER": 1, "SAME_LOWER": 2, "VALID": 3}

EPI_BIAS = 1
EPI_BN = 2
EPI_RESIDUAL = 4
EPI_RELU = 8

ATTR_INT, ATTR_FLOAT, ATTR_INTS, ATTR_STRING = 0, 1, 2, 3


class Options(ctypes.Structure):
    _fields_ = [("precision", ctypes.c_int), ("workspace_bytes", ctypes.c_size_t),
                ("use_cuda_graph", ctypes.c_int), ("wait_timeout_ms", ctypes.c_int)]


class ConvDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in
                ("n", "c", "h", "w", "c_out", "kh", "kw", "stride_h", "stride_w", "pad_top", "pad_left",
                 "pad_bottom", "pad_right", "dil_h", "dil_w", "group")] + [
        ("auto_pad", ctypes.c_int), ("layout", ctypes.c_int), ("epilogue", ctypes.c_int),
        ("precision", ctypes.c_int), ("bn_epsilon", ctypes.c_float)]


class ConvNdDesc(ctypes.Structure):
    _fields_ = [("spatial", ctypes.c_int), ("n", ctypes.c_int64), ("c", ctypes.c_int64),
                ("c_out", ctypes.c_int64), ("group", ctypes.c_int64)] + [
        (f, ctypes.c_int64 * 3) for f in ("in_", "kernel", "stride", "pad_begin", "pad_end", "dilation")] + [
        ("auto_pad", ctypes.c_int), ("relu", ctypes.c_int)]


class Attr(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int), ("i", ctypes.c_int64),
                ("f", ctypes.c_float), ("ints", ctypes.POINTER(ctypes.c_int64)), ("n_ints", ctypes.c_int),
                ("s", ctypes.c_char_p)]


class Node(ctypes.Structure):
    _fields_ = [("op_type", ctypes.c_char_p), ("inputs", ctypes.POINTER(ctypes.c_char_p)),
                ("n_inputs", ctypes.c_int), ("outputs", ctypes.POINTER(ctypes.c_char_p)),
                ("n_outputs", ctypes.c_int), ("attrs", ctypes.POINTER(Attr)), ("n_attrs", ctypes.c_int)]


class TensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.POINTER(ctypes.c_float)),
                ("shape", ctypes.POINTER(ctypes.c_int64)), ("rank", ctypes.c_int)]


class StepProfile(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("ms", ctypes.c_float), ("flops", ctypes.c_double),
                ("bytes", ctypes.c_double)]


STEP_KINDS = {1: "conv_tc", 2: "conv_direct", 3: "gemm", 4: "maxpool", 5: "gap", 6: "add", 7: "relu",
              8: "affine", 9: "convert"}


class GraphStats(ctypes.Structure):
    _fields_ = [("n_nodes_in", ctypes.c_int), ("n_steps", ctypes.c_int), ("n_fused", ctypes.c_int),
                ("kernels_per_run", ctypes.c_int64), ("arena_bytes", ctypes.c_int64),
                ("weight_bytes", ctypes.c_int64), ("captured", ctypes.c_int), ("bf16_tensors", ctypes.c_int)]


class ModelInfo(ctypes.Structure):
    _fields_ = [("ir_version", ctypes.c_int64), ("opset", ctypes.c_int64), ("n_nodes", ctypes.c_int),
                ("n_initializers", ctypes.c_int), ("n_skipped_initializers", ctypes.c_int),
                ("n_skipped_attributes", ctypes.c_int), ("n_inputs", ctypes.c_int), ("n_outputs", ctypes.c_int),
                ("producer_name", ctypes.c_char_p), ("graph_name", ctypes.c_char_p)]


class ShapeInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dims", ctypes.c_int64 * 8), ("rank", ctypes.c_int)]


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i64p = ctypes.POINTER(ctypes.c_int64)
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes)
SIGNATURES = {
    "onnxb200_version": (_int, []),
    "onnxb200_default_options": (None, [ctypes.POINTER(Options)]),
    "onnxb200_create": (_int, [_int, ctypes.POINTER(Options), ctypes.POINTER(_vp)]),
    "onnxb200_destroy": (_int, [_vp]),
    "onnxb200_last_error": (ctypes.c_char_p, [_vp]),
    "onnxb200_status_string": (ctypes.c_char_p, [_int]),
    "onnxb200_set_stream": (_int, [_vp, _vp]),
    "onnxb200_get_stream": (_vp, [_vp]),
    "onnxb200_synchronize": (_int, [_vp]),
    "onnxb200_kernel_launches": (_i64, [_vp]),
    "onnxb200_num_sms": (_int, [_vp]),
    "onnxb200_malloc": (_int, [_vp, ctypes.c_size_t, ctypes.POINTER(_vp)]),
    "onnxb200_free": (_int, [_vp, _vp]),
    "onnxb200_memcpy": (_int, [_vp, _vp, _vp, ctypes.c_size_t, _int]),
    "onnxb200_conv2d_output_shape": (_int, [ctypes.POINTER(ConvDesc), _i64p]),
    "onnxb200_conv2d": (_int, [_vp, ctypes.POINTER(ConvDesc)] + [_vp] * 9),
    "onnxb200_conv_plan_create": (_int, [_vp, ctypes.POINTER(ConvDesc)] + [_vp] * 6 + [ctypes.POINTER(_vp)]),
    "onnxb200_conv_plan_run": (_int, [_vp, _vp, _vp, _vp, _vp]),
    "onnxb200_conv_plan_destroy": (_int, [_vp]),
    "onnxb200_conv_nd_output_shape": (_int, [ctypes.POINTER(ConvNdDesc), _i64p, ctypes.POINTER(_int)]),
    "onnxb200_conv_nd": (_int, [_vp, ctypes.POINTER(ConvNdDesc), _vp, _vp, _vp, _vp]),
    "onnxb200_conv2d_nhwc_noalloc": (_int, [_vp, ctypes.POINTER(ConvDesc)] + [_vp] * 9),
    "onnxb200_matmul_output_shape": (_int, [_i64p, _int, _i64p, _int, _i64p, ctypes.POINTER(_int)]),
    "onnxb200_matmul": (_int, [_vp, _vp, _i64p, _int, _vp, _i64p, _int, _vp, _int, _int, _vp]),
    "onnxb200_gemm": (_int, [_vp, _vp, _vp, _vp, _i64p, _int, _i64, _i64, _i64, _int, _int, _f32, _f32,
                             _int, _int, _vp]),
    "onnxb200_maxpool2d": (_int, [_vp, _int] + [_i64] * 12 + [_int, _vp, _vp, _vp, _i64p]),
    "onnxb200_global_avgpool": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _vp, _vp]),
    "onnxb200_add": (_int, [_vp, _vp, _i64p, _int, _vp, _i64p, _int, _int, _vp]),
    "onnxb200_relu": (_int, [_vp, _vp, _i64, _vp]),
    "onnxb200_batchnorm": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _f32, _vp]),
    "onnxb200_nchw_to_nhwc": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "onnxb200_nhwc_to_nchw": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "onnxb200_graph_build": (_int, [_vp, ctypes.POINTER(Node), _int, ctypes.POINTER(TensorInfo), _int,
                                    ctypes.POINTER(TensorInfo), _int, ctypes.POINTER(ctypes.c_char_p), _int,
                                    ctypes.POINTER(_vp)]),
    "onnxb200_graph_run": (_int, [_vp, _vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "onnxb200_graph_run_host": (_int, [_vp, _vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "onnxb200_graph_run_host_pipelined": (_int, [_vp, _vp, _int, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "onnxb200_graph_output_shape": (_int, [_vp, _int, _i64p, ctypes.POINTER(_int)]),
    "onnxb200_graph_get_stats": (_int, [_vp, ctypes.POINTER(GraphStats)]),
    "onnxb200_multi_build": (_int, [ctypes.POINTER(_int), _int, ctypes.POINTER(Options), ctypes.POINTER(Node), _int,
                                    ctypes.POINTER(TensorInfo), _int, ctypes.POINTER(TensorInfo), _int,
                                    ctypes.POINTER(ctypes.c_char_p), _int, ctypes.POINTER(_vp), ctypes.c_char_p,
                                    ctypes.c_size_t]),
    "onnxb200_multi_run_host": (_int, [_vp, _int, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "onnxb200_multi_get_info": (_int, [_vp, ctypes.POINTER(_int), _i64p, _i64p, ctypes.POINTER(_f32)]),
    "onnxb200_multi_output_shape": (_int, [_vp, _int, _i64p, ctypes.POINTER(_int)]),
    "onnxb200_multi_last_error": (ctypes.c_char_p, [_vp]),
    "onnxb200_multi_destroy": (_int, [_vp]),
    "onnxb200_infer_shapes": (_int, [ctypes.POINTER(Node), _int, ctypes.POINTER(TensorInfo), _int,
                                     ctypes.POINTER(ShapeInfo), _int, ctypes.POINTER(_int), ctypes.c_char_p,
                                     ctypes.c_size_t]),
    "onnxb200_graph_destroy": (_int, [_vp]),
    "onnxb200_graph_profile": (_int, [_vp, _vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                      ctypes.POINTER(StepProfile), _int, ctypes.POINTER(_int)]),
    "onnxb200_model_parse": (_int, [_vp, ctypes.c_size_t, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.c_char_p,
                                    ctypes.c_size_t]),
    "onnxb200_model_load": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.c_char_p, ctypes.c_size_t]),
    "onnxb200_model_get_info": (_int, [_vp, ctypes.POINTER(ModelInfo)]),
    "onnxb200_model_get_nodes": (_int, [_vp, ctypes.POINTER(ctypes.POINTER(Node)), ctypes.POINTER(_int)]),
    "onnxb200_model_get_initializers": (_int, [_vp, ctypes.POINTER(ctypes.POINTER(TensorInfo)),
                                               ctypes.POINTER(_int)]),
    "onnxb200_model_get_inputs": (_int, [_vp, ctypes.POINTER(ctypes.POINTER(TensorInfo)), ctypes.POINTER(_int)]),
    "onnxb200_model_get_outputs": (_int, [_vp, ctypes.POINTER(ctypes.POINTER(ctypes.c_char_p)),
                                          ctypes.POINTER(_int)]),
    "onnxb200_model_destroy": (_int, [_vp]),
    "onnxb200_graph_build_from_model": (_int, [_vp, _vp, ctypes.POINTER(TensorInfo), _int, ctypes.POINTER(_vp)]),
}

_lib = None


def lib():
    """Loads libonnxb200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libonnxb200.so is not built ({LIB_PATH}); run make -C onnx-rs_b200/csrc")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def i64_array(values):
    values = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(values)))(*values)
