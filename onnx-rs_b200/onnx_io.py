""".onnx files in and out.

``load(path_or_bytes)`` parses an ONNX ModelProto with the library's own reader
(``onnxb200_model_parse`` / ``onnxb200_model_load``: OnnxModelLoader,
src/parser/model_loader.rs:27-454, restricted to the main graph) and returns a
:class:`Model` whose nodes, initializers, inputs and outputs are in the same
forms ``Graph`` takes; ``Graph.from_model`` builds the executable graph straight
from it.  Parsing needs no GPU.

``encode_model`` / ``save`` write a node list as a ModelProto -- the writer for
test graphs -- with a hand-written protobuf wire encoder (field numbers of
proto/onnx.proto:65-470, the standard ONNX numbering; external data as ONNX's
key/value entries plus the EXTERNAL data location).
"""
from __future__ import annotations

import ctypes
import os
import struct
from typing import Dict, List, Sequence, Tuple

import numpy as np

from . import _capi as C
from .runtime import raise_for


# ------------------------------------------------------------------ reading
class Model:
    """A parsed model (host memory).  ``nodes`` use the oracle's dict form
    ``{"op", "inputs", "outputs", "attrs"}``; ``initializers`` maps names to
    fp32 arrays; ``inputs`` lists ``(name, shape)`` of the graph inputs that are
    not initializers (-1 for a symbolic dimension); ``outputs`` the output names."""

    def __init__(self, ptr: ctypes.c_void_p):
        self.ptr = ptr
        info = C.ModelInfo()
        self._check(C.lib().onnxb200_model_get_info(ptr, ctypes.byref(info)), "model info")
        self.info = {f: getattr(info, f) for f, _ in C.ModelInfo._fields_}
        for k in ("producer_name", "graph_name"):
            self.info[k] = (self.info[k] or b"").decode()

    @staticmethod
    def _check(code: int, what: str, err: bytes = b""):
        if code != C.OK:
            raise_for(code, f"{what}: {err.decode(errors='replace') or C.lib().onnxb200_status_string(code).decode()}")

    @classmethod
    def from_bytes(cls, data: bytes, base_dir: str | None = None) -> "Model":
        buf = ctypes.create_string_buffer(bytes(data), len(data))
        err = ctypes.create_string_buffer(512)
        ptr = ctypes.c_void_p()
        rc = C.lib().onnxb200_model_parse(buf, len(data), base_dir.encode() if base_dir else None,
                                          ctypes.byref(ptr), err, len(err))
        cls._check(rc, "model parse", err.value)
        return cls(ptr)

    @classmethod
    def from_file(cls, path: str) -> "Model":
        err = ctypes.create_string_buffer(512)
        ptr = ctypes.c_void_p()
        rc = C.lib().onnxb200_model_load(os.fsencode(path), ctypes.byref(ptr), err, len(err))
        cls._check(rc, "model load", err.value)
        return cls(ptr)

    @property
    def nodes(self) -> List[dict]:
        arr = ctypes.POINTER(C.Node)()
        n = ctypes.c_int()
        self._check(C.lib().onnxb200_model_get_nodes(self.ptr, ctypes.byref(arr), ctypes.byref(n)), "model nodes")
        out = []
        for k in range(n.value):
            nd = arr[k]
            attrs = {}
            for j in range(nd.n_attrs):
                a = nd.attrs[j]
                if a.type == C.ATTR_INT:
                    v = int(a.i)
                elif a.type == C.ATTR_FLOAT:
                    v = float(a.f)
                elif a.type == C.ATTR_INTS:
                    v = [int(a.ints[i]) for i in range(a.n_ints)]
                else:
                    v = (a.s or b"").decode()
                attrs[a.name.decode()] = v
            out.append({"op": nd.op_type.decode(),
                        "inputs": [(nd.inputs[i] or b"").decode() for i in range(nd.n_inputs)],
                        "outputs": [nd.outputs[i].decode() for i in range(nd.n_outputs)],
                        "attrs": attrs})
        return out

    @property
    def initializers(self) -> Dict[str, np.ndarray]:
        arr = ctypes.POINTER(C.TensorInfo)()
        n = ctypes.c_int()
        self._check(C.lib().onnxb200_model_get_initializers(self.ptr, ctypes.byref(arr), ctypes.byref(n)),
                    "model initializers")
        out = {}
        for k in range(n.value):
            t = arr[k]
            shape = tuple(int(t.shape[i]) for i in range(t.rank))
            count = int(np.prod(shape)) if shape else 1
            if count:
                data = np.ctypeslib.as_array(t.data, shape=(count,)).copy()
            else:
                data = np.empty(0, np.float32)
            out[t.name.decode()] = data.reshape(shape)
        return out

    @property
    def inputs(self) -> List[Tuple[str, List[int]]]:
        arr = ctypes.POINTER(C.TensorInfo)()
        n = ctypes.c_int()
        self._check(C.lib().onnxb200_model_get_inputs(self.ptr, ctypes.byref(arr), ctypes.byref(n)), "model inputs")
        return [(arr[k].name.decode(), [int(arr[k].shape[i]) for i in range(arr[k].rank)]) for k in range(n.value)]

    @property
    def outputs(self) -> List[str]:
        arr = ctypes.POINTER(ctypes.c_char_p)()
        n = ctypes.c_int()
        self._check(C.lib().onnxb200_model_get_outputs(self.ptr, ctypes.byref(arr), ctypes.byref(n)),
                    "model outputs")
        return [arr[k].decode() for k in range(n.value)]

    def close(self):
        if getattr(self, "ptr", None):
            C.lib().onnxb200_model_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load(source: str | bytes | os.PathLike, base_dir: str | None = None) -> Model:
    """A path (external data resolved next to the file) or the model's bytes."""
    if isinstance(source, (bytes, bytearray, memoryview)):
        return Model.from_bytes(bytes(source), base_dir)
    return Model.from_file(os.fspath(source))


# ------------------------------------------------------------------ writing
def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1  # negative int64 -> ten-byte two's complement
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(num: int, wire: int) -> bytes:
    return _varint((num << 3) | wire)


def _ld(num: int, payload: bytes) -> bytes:
    return _key(num, 2) + _varint(len(payload)) + payload


def _str(num: int, s: str) -> bytes:
    return _ld(num, s.encode())


def _int(num: int, v: int) -> bytes:
    return _key(num, 0) + _varint(int(v))


def _float(num: int, v: float) -> bytes:
    return _key(num, 5) + struct.pack("<f", v)


_ATTR_FLOAT, _ATTR_INT, _ATTR_STRING, _ATTR_INTS = 1, 2, 3, 7  # AttributeProto.AttributeType


def _attribute(name: str, v) -> bytes:
    b = _str(1, name)
    if isinstance(v, str):
        return b + _ld(4, v.encode()) + _int(20, _ATTR_STRING)
    if isinstance(v, float):
        return b + _float(2, v) + _int(20, _ATTR_FLOAT)
    if isinstance(v, (list, tuple)):
        return b + b"".join(_int(8, x) for x in v) + _int(20, _ATTR_INTS)
    return b + _int(3, int(v)) + _int(20, _ATTR_INT)


def _node(nd: dict, index: int) -> bytes:
    b = b"".join(_str(1, s) for s in nd["inputs"])
    b += b"".join(_str(2, s) for s in nd["outputs"])
    b += _str(3, nd.get("name", f"{nd['op']}_{index}"))
    b += _str(4, nd["op"])
    b += b"".join(_ld(5, _attribute(k, v)) for k, v in nd.get("attrs", {}).items())
    return b


def _value_info(name: str, shape: Sequence[int | str] | None) -> bytes:
    tensor_type = _int(1, 1)  # elem_type FLOAT
    if shape is not None:
        dims = b"".join(_ld(1, _str(2, d) if isinstance(d, str) else _int(1, d)) for d in shape)
        tensor_type += _ld(2, dims)
    return _str(1, name) + _ld(2, _ld(1, tensor_type))


def _tensor(name: str, arr: np.ndarray, external: Tuple[str, int] | None) -> bytes:
    a = np.ascontiguousarray(arr, dtype=np.float32)
    b = b"".join(_int(1, d) for d in a.shape) + _int(2, 1) + _str(8, name)
    if external is None:
        return b + _ld(9, a.astype("<f4").tobytes())
    loc, off = external
    for k, v in (("location", loc), ("offset", str(off)), ("length", str(a.nbytes))):
        b += _ld(13, _str(1, k) + _str(2, v))
    return b + _int(14, 1)  # data_location EXTERNAL


def encode_model(nodes: Sequence[dict], initializers: Dict[str, np.ndarray],
                 inputs: Sequence[Tuple[str, Sequence[int | str]]], outputs: Sequence[str | Tuple[str, Sequence]],
                 opset: int = 13, ir_version: int = 8, graph_name: str = "graph",
                 producer: str = "onnx-rs_b200", external: Tuple[str, List[bytes]] | None = None) -> bytes:
    """A ModelProto for a node list.  ``inputs``: (name, shape) with ints or
    symbolic names; ``outputs``: names or (name, shape).  With ``external`` =
    (file name, chunks), initializer bytes are appended to ``chunks`` instead of
    stored inline, and the tensors point into that file."""
    g = b"".join(_ld(1, _node(nd, i)) for i, nd in enumerate(nodes))
    g += _str(2, graph_name)
    off = 0
    for name, arr in initializers.items():
        ext = None
        if external is not None:
            ext = (external[0], off)
            raw = np.ascontiguousarray(arr, dtype=np.float32).astype("<f4").tobytes()
            external[1].append(raw)
            off += len(raw)
        g += _ld(5, _tensor(name, arr, ext))
    g += b"".join(_ld(11, _value_info(n, s)) for n, s in inputs)
    for o in outputs:
        name, shape = (o, None) if isinstance(o, str) else o
        g += _ld(12, _value_info(name, shape))
    m = _int(1, ir_version) + _str(2, producer) + _ld(7, g)
    m += _ld(8, _str(1, "") + _int(2, opset))
    return m


def save(path: str, nodes, initializers, inputs, outputs, external_data: bool = False, **kw) -> None:
    """Writes ``path`` (and ``path + ".data"`` with the initializers when
    ``external_data``)."""
    ext = None
    if external_data:
        ext = (os.path.basename(path) + ".data", [])
    data = encode_model(nodes, initializers, inputs, outputs, external=ext, **kw)
    with open(path, "wb") as f:
        f.write(data)
    if ext is not None:
        with open(path + ".data", "wb") as f:
            for chunk in ext[1]:
                f.write(chunk)
