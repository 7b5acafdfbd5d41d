"""onnx-rs_b200: B200 (sm_100a) implementation of the onnx-rs Conv / MatMul /
Gemm / Conv+BatchNormalization+Relu / Add / MaxPool / GlobalAveragePool path.

All compute lives in ``libonnxb200.so`` (CUDA, tcgen05/TMEM tensor cores) behind
the C ABI of ``include/onnxb200.h``; this package is the host-side mirror of the
reference's operator interface over that ABI.  Import it with
``importlib.import_module("onnx-rs_b200")`` (the directory name has a hyphen).
"""
from . import _capi
from .runtime import (Handle, OnnxB200Error, ValidationError, ExecutionError, UnsupportedFeature,
                      OperationTimeout, ResourceExhausted, InvalidGraph, InvalidOperator, IoError, ProtobufError,
                      InvalidModel)
from .ops import (ExecutionContext, Operator, OperatorRegistry, Conv, ConvPlan, MatMul, Gemm, MaxPool,
                  GlobalAveragePool, Relu, Add, BatchNormalization, Flatten)
from .graph import Graph, MultiGraph, infer_shapes
from . import onnx_io, sharding, synth, workloads

LIB_PATH = _capi.LIB_PATH

__all__ = ["Handle", "OnnxB200Error", "ValidationError", "ExecutionError", "UnsupportedFeature",
           "OperationTimeout", "ResourceExhausted", "InvalidGraph", "InvalidOperator", "ExecutionContext",
           "Operator", "OperatorRegistry", "Conv", "ConvPlan", "MatMul", "Gemm", "MaxPool", "GlobalAveragePool", "Relu",
           "Add", "BatchNormalization", "Flatten", "Graph", "MultiGraph", "infer_shapes", "onnx_io", "synth", "workloads", "LIB_PATH",
           "IoError", "ProtobufError", "InvalidModel"]
