"""Handle, errors and device-buffer plumbing over the C ABI.

Device buffers are torch CUDA tensors (torch is used only for device memory and
streams); every computation runs in libonnxb200.so.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _capi as C


class OnnxB200Error(RuntimeError):
    """Base error; ``code`` is the C-ABI status (src/error.rs:19-66 variants)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class ValidationError(OnnxB200Error):
    pass


class ExecutionError(OnnxB200Error):
    pass


class UnsupportedFeature(OnnxB200Error):
    pass


class OperationTimeout(OnnxB200Error):
    pass


class ResourceExhausted(OnnxB200Error):
    pass


class InvalidGraph(OnnxB200Error):
    pass


class InvalidOperator(OnnxB200Error):
    pass


class IoError(OnnxB200Error):
    pass


class ProtobufError(OnnxB200Error):
    pass


class InvalidModel(OnnxB200Error):
    pass


_ERRORS = {
    C.ERR_VALIDATION: ValidationError, C.ERR_EXECUTION: ExecutionError, C.ERR_UNSUPPORTED: UnsupportedFeature,
    C.ERR_TIMEOUT: OperationTimeout, C.ERR_RESOURCE_EXHAUSTED: ResourceExhausted,
    C.ERR_INVALID_GRAPH: InvalidGraph, C.ERR_INVALID_OPERATOR: InvalidOperator,
    C.ERR_IO: IoError, C.ERR_PROTOBUF: ProtobufError, C.ERR_INVALID_MODEL: InvalidModel,
}


def raise_for(code: int, message: str):
    raise _ERRORS.get(code, OnnxB200Error)(code, message)


class Handle:
    """One GPU context (stream, workspace, status word); ExecutionContext's role.

    By default the handle runs on torch's current stream of ``device`` so that
    torch-allocated buffers are ordered with the library's kernels.
    """

    def __init__(self, device: int = 0, precision: str | int = "3xtf32", workspace_bytes: int = 0,
                 use_cuda_graph: bool = True, wait_timeout_ms: int = 60000, torch_stream: bool = True):
        self.lib = C.lib()
        opts = C.Options()
        self.lib.onnxb200_default_options(ctypes.byref(opts))
        opts.precision = C.PRECISIONS[precision] if isinstance(precision, str) else int(precision)
        opts.workspace_bytes = workspace_bytes
        opts.use_cuda_graph = 1 if use_cuda_graph else 0
        opts.wait_timeout_ms = wait_timeout_ms
        self.device = device
        self.precision = opts.precision
        ptr = ctypes.c_void_p()
        rc = self.lib.onnxb200_create(device, ctypes.byref(opts), ctypes.byref(ptr))
        if rc != 0:
            raise_for(rc, f"onnxb200_create(device={device}) failed: "
                          f"{self.lib.onnxb200_status_string(rc).decode()}")
        self.ptr = ptr
        if torch_stream:
            s = torch.cuda.current_stream(device)
            self.check(self.lib.onnxb200_set_stream(self.ptr, ctypes.c_void_p(s.cuda_stream)))

    def check(self, rc: int, what: str = ""):
        if rc != 0:
            msg = self.lib.onnxb200_last_error(self.ptr).decode() if self.ptr else ""
            raise_for(rc, f"{what}: {msg}" if what else msg)

    def synchronize(self):
        self.check(self.lib.onnxb200_synchronize(self.ptr), "synchronize")

    @property
    def launches(self) -> int:
        return int(self.lib.onnxb200_kernel_launches(self.ptr))

    @property
    def num_sms(self) -> int:
        return int(self.lib.onnxb200_num_sms(self.ptr))

    @property
    def stream_ptr(self) -> int:
        return int(self.lib.onnxb200_get_stream(self.ptr) or 0)

    def close(self):
        if getattr(self, "ptr", None):
            self.lib.onnxb200_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def dptr(t: Optional[torch.Tensor]):
    """Device pointer of a contiguous fp32 CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return ctypes.c_void_p(t.data_ptr())
