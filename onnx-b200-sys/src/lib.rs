//! Bindings to libonnxb200.so, the B200 implementation of onnx-rs's Conv /
//! MatMul / Gemm / Conv+BatchNormalization+Relu / Add / MaxPool /
//! GlobalAveragePool path.  `ffi` is the C ABI of include/onnxb200.h, generated
//! by gen_ffi.py; the types below own its handles and device buffers.
//!
//! Status codes map 1:1 onto the variants of onnx-rs's `crate::error::Error`
//! (src/error.rs:19-66); `Status::code` carries the code and the operator
//! module (ops/b200.rs) converts it.

pub mod ffi;

use std::ffi::CStr;
use std::os::raw::{c_int, c_void};

/// A failed call: the C-ABI status code and the library's message.
#[derive(Debug, Clone)]
pub struct Status {
    pub code: c_int,
    pub message: String,
}

impl std::fmt::Display for Status {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "onnxb200 status {}: {}", self.code, self.message)
    }
}

impl std::error::Error for Status {}

fn status_of(code: c_int, h: *const ffi::Handle) -> Result<(), Status> {
    if code == ffi::ONNXB200_OK {
        return Ok(());
    }
    let msg = unsafe {
        let p = if h.is_null() { ffi::onnxb200_status_string(code) } else { ffi::onnxb200_last_error(h) };
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    Err(Status { code, message: msg })
}

/// One GPU context: a stream, a workspace and a device status word.  The
/// library's handles are used by one host thread at a time, so a `Context` is
/// `Send` but not `Sync`; keep one per worker thread per GPU.
pub struct Context {
    ptr: *mut ffi::Handle,
}

unsafe impl Send for Context {}

impl Context {
    /// `precision`: one of ffi::ONNXB200_PREC_* (3xTF32 is the fp32-accurate default).
    pub fn new(device: i32, precision: c_int) -> Result<Self, Status> {
        unsafe {
            let mut opts: ffi::Options = std::mem::zeroed();
            ffi::onnxb200_default_options(&mut opts);
            opts.precision = precision;
            let mut ptr = std::ptr::null_mut();
            status_of(ffi::onnxb200_create(device, &opts, &mut ptr), std::ptr::null())?;
            Ok(Context { ptr })
        }
    }

    pub fn raw(&self) -> *mut ffi::Handle {
        self.ptr
    }

    /// Turns a status code returned by a call on this context into a Result.
    pub fn check(&self, code: c_int) -> Result<(), Status> {
        status_of(code, self.ptr)
    }

    /// Waits (bounded) for the context's stream and reports device-side failures.
    pub fn synchronize(&self) -> Result<(), Status> {
        self.check(unsafe { ffi::onnxb200_synchronize(self.ptr) })
    }

    /// A device buffer of `len` fp32 elements on this context's GPU.
    pub fn alloc(&self, len: usize) -> Result<DeviceBuffer<'_>, Status> {
        let mut p: *mut c_void = std::ptr::null_mut();
        self.check(unsafe { ffi::onnxb200_malloc(self.ptr, len.max(1) * 4, &mut p) })?;
        Ok(DeviceBuffer { ctx: self, ptr: p, len })
    }

    /// A device buffer holding a copy of `data` (asynchronous on the stream).
    pub fn upload(&self, data: &[f32]) -> Result<DeviceBuffer<'_>, Status> {
        let b = self.alloc(data.len())?;
        if !data.is_empty() {
            self.check(unsafe {
                ffi::onnxb200_memcpy(self.ptr, b.ptr, data.as_ptr() as *const c_void, data.len() * 4,
                                     ffi::ONNXB200_COPY_H2D)
            })?;
        }
        Ok(b)
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe {
            ffi::onnxb200_destroy(self.ptr);
        }
    }
}

/// fp32 device memory owned through a `Context`.
pub struct DeviceBuffer<'a> {
    ctx: &'a Context,
    ptr: *mut c_void,
    len: usize,
}

impl<'a> DeviceBuffer<'a> {
    pub fn len(&self) -> usize {
        self.len
    }
    pub fn is_empty(&self) -> bool {
        self.len == 0
    }
    pub fn as_ptr(&self) -> *const f32 {
        self.ptr as *const f32
    }
    pub fn as_mut_ptr(&self) -> *mut f32 {
        self.ptr as *mut f32
    }
    /// Copies the buffer into `out` and waits for the copy (bounded).
    pub fn download(&self, out: &mut [f32]) -> Result<(), Status> {
        assert_eq!(out.len(), self.len, "download: length mismatch");
        if self.len > 0 {
            self.ctx.check(unsafe {
                ffi::onnxb200_memcpy(self.ctx.ptr, out.as_mut_ptr() as *mut c_void, self.ptr, self.len * 4,
                                     ffi::ONNXB200_COPY_D2H)
            })?;
        }
        self.ctx.synchronize()
    }
}

impl<'a> Drop for DeviceBuffer<'a> {
    fn drop(&mut self) {
        unsafe {
            ffi::onnxb200_free(self.ctx.ptr, self.ptr);
        }
    }
}
