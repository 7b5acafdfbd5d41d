"""Graph API: the ExecutionEngine (src/execution/engine.rs:75-231) of this path.

``Graph(handle, nodes, initializers, inputs, outputs)`` hands an ONNX-style node
list to ``onnxb200_graph_build`` (fusion, NHWC weight packing, one activation
arena, CUDA-graph capture on replay) and runs it on device or host buffers.
Nodes use the same dict form as the oracle: ``{"op", "inputs", "outputs", "attrs"}``.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Sequence, Tuple

import numpy as np
import torch

from . import _capi as C
from .runtime import Handle, dptr


def _c_node(nd: dict, keep: list) -> C.Node:
    ins = [s.encode() if s else b"" for s in nd["inputs"]]
    outs = [s.encode() for s in nd["outputs"]]
    in_arr = (ctypes.c_char_p * max(1, len(ins)))(*ins)
    out_arr = (ctypes.c_char_p * max(1, len(outs)))(*outs)
    attrs = []
    for k, v in nd.get("attrs", {}).items():
        a = C.Attr()
        a.name = k.encode()
        keep.append(a.name)
        if isinstance(v, str):
            a.type = C.ATTR_STRING
            a.s = v.encode()
            keep.append(a.s)
        elif isinstance(v, float):
            a.type = C.ATTR_FLOAT
            a.f = v
        elif isinstance(v, (list, tuple)):
            a.type = C.ATTR_INTS
            arr = C.i64_array(v)
            keep.append(arr)
            a.ints = ctypes.cast(arr, ctypes.POINTER(ctypes.c_int64))
            a.n_ints = len(v)
        else:
            a.type = C.ATTR_INT
            a.i = int(v)
        attrs.append(a)
    attr_arr = (C.Attr * max(1, len(attrs)))(*attrs)
    keep += [ins, outs, in_arr, out_arr, attr_arr]
    n = C.Node()
    n.op_type = nd["op"].encode()
    keep.append(n.op_type)
    n.inputs = ctypes.cast(in_arr, ctypes.POINTER(ctypes.c_char_p))
    n.n_inputs = len(ins)
    n.outputs = ctypes.cast(out_arr, ctypes.POINTER(ctypes.c_char_p))
    n.n_outputs = len(outs)
    n.attrs = ctypes.cast(attr_arr, ctypes.POINTER(C.Attr))
    n.n_attrs = len(attrs)
    return n


def _c_shapes(shapes: Dict[str, Sequence[int]], keep: list):
    arr = (C.TensorInfo * max(1, len(shapes)))()
    for i, (name, shp) in enumerate(shapes.items()):
        t = arr[i]
        t.name = name.encode()
        keep.append(t.name)
        dims = C.i64_array(shp)
        keep.append(dims)
        t.shape = ctypes.cast(dims, ctypes.POINTER(ctypes.c_int64))
        t.rank = len(shp)
    return arr


def infer_shapes(nodes: Sequence[dict], known: Dict[str, Sequence[int]]) -> Dict[str, List[int]]:
    """Shapes of every node output of a node list, without building a graph
    (``onnxb200_infer_shapes``; the planner's infer_node_output_shapes,
    src/memory/planner.rs:908-960).  ``known`` maps initializer and graph-input
    names to their shapes.  Host only: no handle, no GPU."""
    from .runtime import raise_for
    keep: list = []
    cnodes = (C.Node * max(1, len(nodes)))(*[_c_node(nd, keep) for nd in nodes])
    ck = _c_shapes(dict(known), keep)
    n_out = sum(len(nd["outputs"]) for nd in nodes)
    out = (C.ShapeInfo * max(1, n_out))()
    n = ctypes.c_int()
    err = ctypes.create_string_buffer(512)
    rc = C.lib().onnxb200_infer_shapes(cnodes, len(nodes), ck, len(known), out, n_out, ctypes.byref(n), err, 512)
    if rc:
        raise_for(rc, err.value.decode(errors="replace"))
    return {out[i].name.decode(): [int(out[i].dims[d]) for d in range(out[i].rank)] for i in range(n.value)}


class Graph:
    def __init__(self, handle: Handle, nodes: Sequence[dict], initializers: Dict[str, np.ndarray],
                 inputs: Sequence[Tuple[str, Sequence[int]]], outputs: Sequence[str]):
        self.handle = handle
        self.input_specs = [(n, list(s)) for n, s in inputs]
        self.output_names = list(outputs)
        keep: list = []
        cnodes = (C.Node * max(1, len(nodes)))(*[_c_node(nd, keep) for nd in nodes])
        inits = []
        for name, arr in initializers.items():
            a = np.ascontiguousarray(arr, dtype=np.float32)
            keep.append(a)
            t = C.TensorInfo()
            t.name = name.encode()
            keep.append(t.name)
            t.data = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            shp = C.i64_array(a.shape)
            keep.append(shp)
            t.shape = ctypes.cast(shp, ctypes.POINTER(ctypes.c_int64))
            t.rank = a.ndim
            inits.append(t)
        init_arr = (C.TensorInfo * max(1, len(inits)))(*inits)
        ins = []
        for name, shape in self.input_specs:
            t = C.TensorInfo()
            t.name = name.encode()
            keep.append(t.name)
            shp = C.i64_array(shape)
            keep.append(shp)
            t.shape = ctypes.cast(shp, ctypes.POINTER(ctypes.c_int64))
            t.rank = len(shape)
            ins.append(t)
        in_arr = (C.TensorInfo * max(1, len(ins)))(*ins)
        onames = [o.encode() for o in outputs]
        out_arr = (ctypes.c_char_p * max(1, len(onames)))(*onames)
        ptr = ctypes.c_void_p()
        handle.check(C.lib().onnxb200_graph_build(handle.ptr, cnodes, len(nodes), init_arr, len(inits), in_arr,
                                                  len(ins), out_arr, len(onames), ctypes.byref(ptr)), "graph build")
        self.ptr = ptr
        self._read_output_shapes()

    def _read_output_shapes(self):
        self.output_shapes = []
        for i in range(len(self.output_names)):
            shp = C.i64_array([0] * 8)
            r = ctypes.c_int()
            self.handle.check(C.lib().onnxb200_graph_output_shape(self.ptr, i, shp, ctypes.byref(r)))
            self.output_shapes.append([int(v) for v in shp[:r.value]])

    @classmethod
    def from_model(cls, handle: Handle, model, input_shapes: Dict[str, Sequence[int]] | None = None) -> "Graph":
        """onnxb200_graph_build_from_model: the graph of a parsed .onnx model
        (``onnx_io.load``); ``input_shapes`` fixes symbolic input dimensions."""
        input_shapes = dict(input_shapes or {})
        keep: list = []
        over = []
        for name, shape in input_shapes.items():
            t = C.TensorInfo()
            t.name = name.encode()
            shp = C.i64_array(shape)
            keep += [t.name, shp]
            t.shape = ctypes.cast(shp, ctypes.POINTER(ctypes.c_int64))
            t.rank = len(shape)
            over.append(t)
        arr = (C.TensorInfo * max(1, len(over)))(*over)
        ptr = ctypes.c_void_p()
        handle.check(C.lib().onnxb200_graph_build_from_model(handle.ptr, model.ptr, arr, len(over), ctypes.byref(ptr)),
                     "graph build from model")
        g = cls.__new__(cls)
        g.handle = handle
        g.input_specs = [(n, list(input_shapes.get(n, s))) for n, s in model.inputs]
        g.output_names = model.outputs
        g.ptr = ptr
        g._read_output_shapes()
        return g

    def stats(self) -> dict:
        s = C.GraphStats()
        self.handle.check(C.lib().onnxb200_graph_get_stats(self.ptr, ctypes.byref(s)))
        return {f: getattr(s, f) for f, _ in C.GraphStats._fields_}

    def alloc_outputs(self, device) -> List[torch.Tensor]:
        return [torch.empty(s, dtype=torch.float32, device=device) for s in self.output_shapes]

    def run(self, inputs: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor] | None = None) -> List[torch.Tensor]:
        """Asynchronous run on device tensors (NCHW)."""
        if outputs is None:
            outputs = self.alloc_outputs(inputs[0].device)
        for t, (name, shape) in zip(inputs, self.input_specs):
            if list(t.shape) != shape:
                raise ValueError(f"input {name}: expected shape {shape}, got {list(t.shape)}")
        iarr = (ctypes.c_void_p * max(1, len(inputs)))(*[t.data_ptr() for t in inputs])
        oarr = (ctypes.c_void_p * max(1, len(outputs)))(*[t.data_ptr() for t in outputs])
        self.handle.check(C.lib().onnxb200_graph_run(self.handle.ptr, self.ptr, iarr, oarr), "graph run")
        return list(outputs)

    def run_host(self, inputs: Sequence[np.ndarray | torch.Tensor],
                 outputs: Sequence[np.ndarray | torch.Tensor] | None = None):
        """Host buffers in and out (copies inside); returns after the results are on the host."""
        ins = [np.ascontiguousarray(x, dtype=np.float32) if isinstance(x, np.ndarray) else x for x in inputs]
        if outputs is None:
            outputs = [np.empty(s, np.float32) for s in self.output_shapes]

        def addr(t):
            return t.ctypes.data if isinstance(t, np.ndarray) else t.data_ptr()

        iarr = (ctypes.c_void_p * max(1, len(ins)))(*[addr(t) for t in ins])
        oarr = (ctypes.c_void_p * max(1, len(outputs)))(*[addr(t) for t in outputs])
        self.handle.check(C.lib().onnxb200_graph_run_host(self.handle.ptr, self.ptr, iarr, oarr), "graph run_host")
        return list(outputs)

    def run_host_pipelined(self, batches: Sequence[Sequence[np.ndarray | torch.Tensor]],
                           outputs: Sequence[Sequence[np.ndarray | torch.Tensor]] | None = None):
        """Several host batches in a row (onnxb200_graph_run_host_pipelined): each
        batch's input copy overlaps the previous batch's compute.  Host buffers
        should be pinned (torch ``pin_memory()``) for the copies to overlap."""
        def addr(t):
            return t.ctypes.data if isinstance(t, np.ndarray) else t.data_ptr()

        ins = [[np.ascontiguousarray(x, dtype=np.float32) if isinstance(x, np.ndarray) else x for x in b]
               for b in batches]
        if outputs is None:
            outputs = [[np.empty(s, np.float32) for s in self.output_shapes] for _ in ins]
        flat_in = [addr(t) for b in ins for t in b]
        flat_out = [addr(t) for b in outputs for t in b]
        iarr = (ctypes.c_void_p * max(1, len(flat_in)))(*flat_in)
        oarr = (ctypes.c_void_p * max(1, len(flat_out)))(*flat_out)
        self.handle.check(C.lib().onnxb200_graph_run_host_pipelined(self.handle.ptr, self.ptr, len(ins), iarr, oarr),
                          "graph run_host_pipelined")
        return [list(o) for o in outputs]

    def profile(self, inputs: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor] | None = None) -> List[dict]:
        """One eager run with CUDA events around every step; returns per-step
        {kind, ms, flops, bytes} (algorithmic work)."""
        if outputs is None:
            outputs = self.alloc_outputs(inputs[0].device)
        iarr = (ctypes.c_void_p * max(1, len(inputs)))(*[t.data_ptr() for t in inputs])
        oarr = (ctypes.c_void_p * max(1, len(outputs)))(*[t.data_ptr() for t in outputs])
        cap = 4096
        prof = (C.StepProfile * cap)()
        n = ctypes.c_int()
        self.handle.check(C.lib().onnxb200_graph_profile(self.handle.ptr, self.ptr, iarr, oarr, prof, cap,
                                                         ctypes.byref(n)), "graph profile")
        return [{"kind": C.STEP_KINDS.get(p.kind, str(p.kind)), "ms": p.ms, "flops": p.flops, "bytes": p.bytes}
                for p in prof[:min(n.value, cap)]]

    def close(self):
        if getattr(self, "ptr", None):
            C.lib().onnxb200_graph_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MultiGraph:
    """Batch-sharded replicas of one graph on several GPUs of this process
    (``onnxb200_multi_build``): every input is split along its first dimension
    into contiguous slices, one per device, each device holds a full copy of
    the packed weights, and there is no collective.  ``run_host`` drives one
    host thread per device; each copies its rows in, replays its graph and
    copies its rows of the outputs into disjoint rows of the host outputs."""

    def __init__(self, devices: Sequence[int], nodes: Sequence[dict], initializers: Dict[str, np.ndarray],
                 inputs: Sequence[Tuple[str, Sequence[int]]], outputs: Sequence[str],
                 precision: str | int = "3xtf32", use_cuda_graph: bool = True):
        from .runtime import raise_for
        self.lib = C.lib()
        opts = C.Options()
        self.lib.onnxb200_default_options(ctypes.byref(opts))
        opts.precision = C.PRECISIONS[precision] if isinstance(precision, str) else int(precision)
        opts.use_cuda_graph = 1 if use_cuda_graph else 0
        keep: list = []
        cnodes = (C.Node * max(1, len(nodes)))(*[_c_node(nd, keep) for nd in nodes])
        arrs = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in initializers.items()}
        inits = (C.TensorInfo * max(1, len(arrs)))()
        for i, (name, a) in enumerate(arrs.items()):
            t = inits[i]
            t.name = name.encode()
            shp = C.i64_array(a.shape)
            keep += [t.name, shp]
            t.data = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            t.shape = ctypes.cast(shp, ctypes.POINTER(ctypes.c_int64))
            t.rank = a.ndim
        ins = _c_shapes({n: list(s) for n, s in inputs}, keep)
        onames = [o.encode() for o in outputs]
        out_arr = (ctypes.c_char_p * max(1, len(onames)))(*onames)
        devs = (ctypes.c_int * len(devices))(*devices)
        err = ctypes.create_string_buffer(512)
        ptr = ctypes.c_void_p()
        rc = self.lib.onnxb200_multi_build(devs, len(devices), ctypes.byref(opts), cnodes, len(nodes), inits,
                                           len(arrs), ins, len(inputs), out_arr, len(onames), ctypes.byref(ptr),
                                           err, 512)
        if rc:
            raise_for(rc, err.value.decode(errors="replace"))
        self.ptr = ptr
        self.devices = list(devices)
        self.input_specs = [(n, list(s)) for n, s in inputs]
        self.output_shapes = []
        for i in range(len(onames)):
            shp = C.i64_array([0] * 8)
            r = ctypes.c_int()
            self.lib.onnxb200_multi_output_shape(self.ptr, i, shp, ctypes.byref(r))
            self.output_shapes.append([int(v) for v in shp[:r.value]])

    def run_host(self, batches: Sequence[Sequence[np.ndarray | torch.Tensor]],
                 outputs: Sequence[Sequence[np.ndarray | torch.Tensor]] | None = None):
        """Runs full batches from host buffers (pinned for overlapped copies);
        returns the host outputs, one list per batch."""
        from .runtime import raise_for

        def addr(t):
            return t.ctypes.data if isinstance(t, np.ndarray) else t.data_ptr()

        ins = [[np.ascontiguousarray(x, dtype=np.float32) if isinstance(x, np.ndarray) else x for x in b]
               for b in batches]
        for b in ins:
            for t, (name, shape) in zip(b, self.input_specs):
                if list(t.shape) != shape:
                    raise ValueError(f"input {name}: expected shape {shape}, got {list(t.shape)}")
        if outputs is None:
            outputs = [[np.empty(s, np.float32) for s in self.output_shapes] for _ in ins]
        flat_in = [addr(t) for b in ins for t in b]
        flat_out = [addr(t) for b in outputs for t in b]
        iarr = (ctypes.c_void_p * max(1, len(flat_in)))(*flat_in)
        oarr = (ctypes.c_void_p * max(1, len(flat_out)))(*flat_out)
        rc = self.lib.onnxb200_multi_run_host(self.ptr, len(ins), iarr, oarr)
        if rc:
            raise_for(rc, self.lib.onnxb200_multi_last_error(self.ptr).decode(errors="replace"))
        return [list(o) for o in outputs]

    def info(self) -> dict:
        n = len(self.devices)
        nd = ctypes.c_int()
        b = ctypes.c_int64()
        lo = (ctypes.c_int64 * n)()
        ms = (ctypes.c_float * n)()
        self.lib.onnxb200_multi_get_info(self.ptr, ctypes.byref(nd), ctypes.byref(b), lo, ms)
        return {"n_devices": nd.value, "batch": b.value, "slice_begin": list(lo), "last_run_ms": list(ms)}

    def close(self):
        if getattr(self, "ptr", None):
            self.lib.onnxb200_multi_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
