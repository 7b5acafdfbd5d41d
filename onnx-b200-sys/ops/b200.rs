//! B200 operators behind onnx-rs's `Operator` trait (src/ops/registry.rs:14-27).
//!
//! This file is the module a maintainer adds to the onnx-rs crate as
//! `src/ops/b200.rs` (with `pub mod b200;` in src/ops/mod.rs and
//! `onnx-b200-sys = { path = "..." }` under [dependencies]).  Each operator
//! keeps the reference operator's contract: `compute` borrows host `Tensor`s and
//! replaces `outputs[0]` wholesale with a new tensor (conv.rs:199-200,
//! matmul.rs:76-77); errors are `crate::error::Error` variants; instances are
//! immutable and may be called from several rayon workers at once, each worker
//! thread using its own GPU context.
//!
//! Unlike the reference operators (whose `compute` uses struct fields and
//! ignores the node, e.g. Conv at conv.rs:156-203 and Gemm at gemm.rs:35-38),
//! these are built from the node's ONNX attributes (`from_node`), so
//! `create_b200_operator_for_node` is the factory to call from
//! `OperatorRegistry::create_operator_for_node`.
//!
//! Execution-context options read here:
//!   "b200.device"     GPU ordinal (default 0)
//!   "b200.precision"  "3xtf32" (default, fp32-accurate) | "tf32" | "bf16" | "fp32"

use std::cell::RefCell;
use std::collections::HashMap;

use ndarray::{ArrayD, IxDyn};
use onnx_b200_sys::{self as sys, ffi};

use crate::error::{Error, Result};
use crate::model::{Attribute, Node};
use crate::ops::registry::{ExecutionContext, Operator, OperatorRegistry};
use crate::ops::tensor::{DataType, Shape, Tensor};

// ---------------------------------------------------------------- plumbing

/// crate::error::Error for a C-ABI status (the codes are defined to match the
/// variants one to one, src/error.rs:19-66).
fn to_error(s: sys::Status) -> Error {
    let m = s.message;
    match s.code {
        ffi::ONNXB200_ERR_VALIDATION => Error::ValidationError(m),
        ffi::ONNXB200_ERR_UNSUPPORTED => Error::UnsupportedFeature(m),
        ffi::ONNXB200_ERR_TIMEOUT => Error::OperationTimeout(m),
        ffi::ONNXB200_ERR_RESOURCE_EXHAUSTED => Error::ResourceExhausted(m),
        ffi::ONNXB200_ERR_INVALID_GRAPH => Error::InvalidGraph(m),
        ffi::ONNXB200_ERR_INVALID_OPERATOR => Error::InvalidOperator(m),
        ffi::ONNXB200_ERR_CANCELLED => Error::ExecutionCancelled(m),
        ffi::ONNXB200_ERR_IO => Error::IoError(m),
        ffi::ONNXB200_ERR_PROTOBUF => Error::ProtobufError(m),
        ffi::ONNXB200_ERR_INVALID_MODEL => Error::InvalidModel(m),
        _ => Error::ExecutionError(m),
    }
}

fn option<'a>(ctx: &'a ExecutionContext, key: &str) -> Option<&'a str> {
    ctx.options.get(key).map(|s| s.as_str())
}

fn precision_of(ctx: &ExecutionContext) -> Result<i32> {
    match option(ctx, "b200.precision").unwrap_or("3xtf32") {
        "3xtf32" => Ok(ffi::ONNXB200_PREC_3XTF32),
        "tf32" => Ok(ffi::ONNXB200_PREC_TF32),
        "bf16" => Ok(ffi::ONNXB200_PREC_BF16),
        "fp32" => Ok(ffi::ONNXB200_PREC_FP32),
        p => Err(Error::ValidationError(format!("b200.precision: unknown precision {}", p))),
    }
}

thread_local! {
    // One GPU context per rayon worker thread and device (the library's handles
    // are used by one thread at a time).
    static CONTEXTS: RefCell<HashMap<i32, sys::Context>> = RefCell::new(HashMap::new());
}

/// Runs `f` with this thread's context on the device the options name.
fn with_context<R>(ctx: &ExecutionContext, f: impl FnOnce(&sys::Context) -> Result<R>) -> Result<R> {
    let device: i32 = option(ctx, "b200.device")
        .unwrap_or("0")
        .parse()
        .map_err(|_| Error::ValidationError("b200.device: not an integer".into()))?;
    CONTEXTS.with(|c| {
        let mut map = c.borrow_mut();
        if !map.contains_key(&device) {
            let context = sys::Context::new(device, ffi::ONNXB200_PREC_3XTF32).map_err(to_error)?;
            map.insert(device, context);
        }
        f(map.get(&device).expect("context just inserted"))
    })
}

fn data_of(t: &Tensor) -> Result<&[f32]> {
    t.data
        .as_slice()
        .ok_or_else(|| Error::ValidationError("tensor data is not contiguous in standard order".into()))
}

fn dims_i64(shape: &Shape) -> Vec<i64> {
    shape.iter().map(|&d| d as i64).collect()
}

fn new_tensor(shape: Vec<usize>, data: Vec<f32>) -> Result<Tensor> {
    let arr = ArrayD::from_shape_vec(IxDyn(&shape), data)
        .map_err(|e| Error::ExecutionError(format!("output tensor: {}", e)))?;
    Tensor::from_ndarray_simple(arr, DataType::Float32)
}

fn ints(node: &Node, name: &str) -> Option<Vec<i64>> {
    match node.attributes.get(name) {
        Some(Attribute::Ints(v)) => Some(v.clone()),
        _ => None,
    }
}

fn int(node: &Node, name: &str, default: i64) -> i64 {
    match node.attributes.get(name) {
        Some(Attribute::Int(v)) => *v,
        _ => default,
    }
}

fn float(node: &Node, name: &str, default: f32) -> f32 {
    match node.attributes.get(name) {
        Some(Attribute::Float(v)) => *v,
        _ => default,
    }
}

fn string(node: &Node, name: &str, default: &str) -> String {
    match node.attributes.get(name) {
        Some(Attribute::String(v)) => v.clone(),
        _ => default.to_string(),
    }
}

fn need_inputs(inputs: &[&Tensor], n: usize, op: &str) -> Result<()> {
    if inputs.len() < n {
        return Err(Error::ValidationError(format!("{} requires at least {} inputs, got {}", op, n, inputs.len())));
    }
    Ok(())
}

fn need_output(outputs: &[Tensor], op: &str) -> Result<()> {
    if outputs.is_empty() {
        return Err(Error::ValidationError(format!("{} requires at least 1 output, got 0", op)));
    }
    Ok(())
}

fn known(input_shapes: &[Option<Shape>], i: usize, op: &str) -> Result<Shape> {
    input_shapes
        .get(i)
        .cloned()
        .flatten()
        .ok_or_else(|| Error::ValidationError(format!("{}: shape of input {} is unknown", op, i)))
}

// ---------------------------------------------------------------- Conv

/// Conv (src/ops/nn/conv.rs:156-323) on the tcgen05 implicit-GEMM path (2-D)
/// or onnxb200_conv_nd (1-D on the tensor cores, 3-D on CUDA cores).
#[derive(Debug, Clone, Default)]
pub struct B200Conv {
    pub strides: Vec<i64>,
    pub pads: Vec<i64>,
    pub dilations: Vec<i64>,
    pub group: i64,
    pub auto_pad: i32,
}

impl B200Conv {
    pub fn from_node(node: &Node) -> Result<Self> {
        let auto_pad = match string(node, "auto_pad", "NOTSET").as_str() {
            "NOTSET" => ffi::ONNXB200_AUTOPAD_NOTSET,
            "SAME_UPPER" => ffi::ONNXB200_AUTOPAD_SAME_UPPER,
            "SAME_LOWER" => ffi::ONNXB200_AUTOPAD_SAME_LOWER,
            "VALID" => ffi::ONNXB200_AUTOPAD_VALID,
            p => return Err(Error::ValidationError(format!("Conv: unknown auto_pad {}", p))),
        };
        Ok(B200Conv {
            strides: ints(node, "strides").unwrap_or_default(),
            pads: ints(node, "pads").unwrap_or_default(),
            dilations: ints(node, "dilations").unwrap_or_default(),
            group: int(node, "group", 1),
            auto_pad,
        })
    }

    fn desc2d(&self, x: &Shape, w: &Shape, epilogue: i32, precision: i32) -> Result<ffi::ConvDesc> {
        if x.len() != 4 || w.len() != 4 {
            return Err(Error::ValidationError("Conv: 2-D descriptor needs rank-4 input and weight".into()));
        }
        let at = |v: &Vec<i64>, i: usize, d: i64| v.get(i).copied().unwrap_or(d);
        let mut d: ffi::ConvDesc = unsafe { std::mem::zeroed() };
        d.n = x[0] as i64;
        d.c = x[1] as i64;
        d.h = x[2] as i64;
        d.w = x[3] as i64;
        d.c_out = w[0] as i64;
        d.kh = w[2] as i64;
        d.kw = w[3] as i64;
        d.stride_h = at(&self.strides, 0, 1);
        d.stride_w = at(&self.strides, 1, d.stride_h);
        d.pad_top = at(&self.pads, 0, 0);
        d.pad_left = at(&self.pads, 1, 0);
        d.pad_bottom = at(&self.pads, 2, d.pad_top);
        d.pad_right = at(&self.pads, 3, d.pad_left);
        d.dil_h = at(&self.dilations, 0, 1);
        d.dil_w = at(&self.dilations, 1, d.dil_h);
        d.group = if self.group > 0 { self.group } else { 1 };
        d.auto_pad = self.auto_pad;
        d.layout = ffi::ONNXB200_LAYOUT_NCHW;
        d.epilogue = epilogue;
        d.precision = precision;
        d.bn_epsilon = 1e-5;
        Ok(d)
    }

    fn desc_nd(&self, x: &Shape, w: &Shape) -> Result<ffi::ConvNdDesc> {
        let sp = x.len() as i64 - 2;
        if !(1..=3).contains(&sp) || w.len() != x.len() {
            return Err(Error::UnsupportedFeature(format!("Conv: {} spatial dims", sp)));
        }
        let sp = sp as usize;
        let mut d: ffi::ConvNdDesc = unsafe { std::mem::zeroed() };
        d.spatial = sp as i32;
        d.n = x[0] as i64;
        d.c = x[1] as i64;
        d.c_out = w[0] as i64;
        d.group = self.group;
        for i in 0..sp {
            d.in_[i] = x[2 + i] as i64;
            d.kernel[i] = w[2 + i] as i64;
            d.stride[i] = self.strides.get(i).copied().unwrap_or(1);
            d.dilation[i] = self.dilations.get(i).copied().unwrap_or(1);
            d.pad_begin[i] = self.pads.get(i).copied().unwrap_or(0);
            d.pad_end[i] = self.pads.get(sp + i).copied().unwrap_or(d.pad_begin[i]);
        }
        d.auto_pad = self.auto_pad;
        Ok(d)
    }
}

impl Operator for B200Conv {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 2, "Conv")?;
        need_output(outputs, "Conv")?;
        let (x, w) = (inputs[0], inputs[1]);
        let b = inputs.get(2).copied();
        let precision = precision_of(ctx)?;
        let result = with_context(ctx, |c| {
            let xd = c.upload(data_of(x)?).map_err(to_error)?;
            let wd = c.upload(data_of(w)?).map_err(to_error)?;
            let bd = match b {
                Some(t) => Some(c.upload(data_of(t)?).map_err(to_error)?),
                None => None,
            };
            let bptr = bd.as_ref().map_or(std::ptr::null(), |t| t.as_ptr());
            if x.shape.len() == 4 {
                let epi = if b.is_some() { ffi::ONNXB200_EPI_BIAS } else { 0 };
                let d = self.desc2d(&x.shape, &w.shape, epi, precision)?;
                let mut o = [0i64; 4];
                c.check(unsafe { ffi::onnxb200_conv2d_output_shape(&d, o.as_mut_ptr()) }).map_err(to_error)?;
                let shape: Vec<usize> = o.iter().map(|&v| v as usize).collect();
                let yd = c.alloc(shape.iter().product()).map_err(to_error)?;
                let nul = std::ptr::null();
                c.check(unsafe {
                    ffi::onnxb200_conv2d(c.raw(), &d, xd.as_ptr(), wd.as_ptr(), bptr, nul, nul, nul, nul, nul,
                                         yd.as_mut_ptr())
                })
                .map_err(to_error)?;
                let mut host = vec![0f32; yd.len()];
                yd.download(&mut host).map_err(to_error)?;
                new_tensor(shape, host)
            } else {
                let d = self.desc_nd(&x.shape, &w.shape)?;
                let mut o = [0i64; 5];
                let mut rank = 0;
                c.check(unsafe { ffi::onnxb200_conv_nd_output_shape(&d, o.as_mut_ptr(), &mut rank) })
                    .map_err(to_error)?;
                let shape: Vec<usize> = o[..rank as usize].iter().map(|&v| v as usize).collect();
                let yd = c.alloc(shape.iter().product()).map_err(to_error)?;
                c.check(unsafe {
                    ffi::onnxb200_conv_nd(c.raw(), &d, xd.as_ptr(), wd.as_ptr(), bptr, yd.as_mut_ptr())
                })
                .map_err(to_error)?;
                let mut host = vec![0f32; yd.len()];
                yd.download(&mut host).map_err(to_error)?;
                new_tensor(shape, host)
            }
        })?;
        outputs[0] = result;
        Ok(())
    }

    fn output_shapes(&self, node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        let conv = B200Conv::from_node(node)?;
        let x = known(input_shapes, 0, "Conv")?;
        let w = known(input_shapes, 1, "Conv")?;
        let shape = if x.len() == 4 {
            let d = conv.desc2d(&x, &w, 0, ffi::ONNXB200_PREC_DEFAULT)?;
            let mut o = [0i64; 4];
            let rc = unsafe { ffi::onnxb200_conv2d_output_shape(&d, o.as_mut_ptr()) };
            if rc != ffi::ONNXB200_OK {
                return Err(Error::ValidationError("Conv: invalid attributes for these shapes".into()));
            }
            o.iter().map(|&v| v as usize).collect()
        } else {
            let d = conv.desc_nd(&x, &w)?;
            let mut o = [0i64; 5];
            let mut rank = 0;
            let rc = unsafe { ffi::onnxb200_conv_nd_output_shape(&d, o.as_mut_ptr(), &mut rank) };
            if rc != ffi::ONNXB200_OK {
                return Err(Error::ValidationError("Conv: invalid attributes for these shapes".into()));
            }
            o[..rank as usize].iter().map(|&v| v as usize).collect()
        };
        Ok(vec![Some(shape)])
    }

    fn validate(&self, node: &Node) -> Result<()> {
        if node.inputs.len() < 2 {
            return Err(Error::ValidationError("Conv requires at least 2 inputs".into()));
        }
        B200Conv::from_node(node).map(|_| ())
    }
}

// ---------------------------------------------------------------- MatMul

/// MatMul (src/ops/math/matmul.rs:124-279): numpy-broadcast batched MatMul.
#[derive(Debug, Clone, Default)]
pub struct B200MatMul;

impl Operator for B200MatMul {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 2, "MatMul")?;
        need_output(outputs, "MatMul")?;
        let (a, b) = (inputs[0], inputs[1]);
        let precision = precision_of(ctx)?;
        let (asz, bsz) = (dims_i64(&a.shape), dims_i64(&b.shape));
        let mut o = [0i64; 16];
        let mut rank = 0;
        let rc = unsafe {
            ffi::onnxb200_matmul_output_shape(asz.as_ptr(), asz.len() as i32, bsz.as_ptr(), bsz.len() as i32,
                                              o.as_mut_ptr(), &mut rank)
        };
        if rc != ffi::ONNXB200_OK {
            return Err(Error::ValidationError(format!("MatMul: incompatible shapes {:?} x {:?}", a.shape, b.shape)));
        }
        let shape: Vec<usize> = o[..rank as usize].iter().map(|&v| v as usize).collect();
        outputs[0] = with_context(ctx, |c| {
            let ad = c.upload(data_of(a)?).map_err(to_error)?;
            let bd = c.upload(data_of(b)?).map_err(to_error)?;
            let yd = c.alloc(shape.iter().product()).map_err(to_error)?;
            c.check(unsafe {
                ffi::onnxb200_matmul(c.raw(), ad.as_ptr(), asz.as_ptr(), asz.len() as i32, bd.as_ptr(),
                                     bsz.as_ptr(), bsz.len() as i32, std::ptr::null(), 0, precision,
                                     yd.as_mut_ptr())
            })
            .map_err(to_error)?;
            let mut host = vec![0f32; yd.len()];
            yd.download(&mut host).map_err(to_error)?;
            new_tensor(shape.clone(), host)
        })?;
        Ok(())
    }

    fn output_shapes(&self, _node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        let (a, b) = (dims_i64(&known(input_shapes, 0, "MatMul")?), dims_i64(&known(input_shapes, 1, "MatMul")?));
        let mut o = [0i64; 16];
        let mut rank = 0;
        let rc = unsafe {
            ffi::onnxb200_matmul_output_shape(a.as_ptr(), a.len() as i32, b.as_ptr(), b.len() as i32,
                                              o.as_mut_ptr(), &mut rank)
        };
        if rc != ffi::ONNXB200_OK {
            return Err(Error::ValidationError("MatMul: incompatible shapes".into()));
        }
        Ok(vec![Some(o[..rank as usize].iter().map(|&v| v as usize).collect())])
    }

    fn validate(&self, node: &Node) -> Result<()> {
        if node.inputs.len() != 2 {
            return Err(Error::ValidationError("MatMul requires 2 inputs".into()));
        }
        Ok(())
    }
}

// ---------------------------------------------------------------- Gemm

/// Gemm (src/ops/math/gemm.rs:17-406) with alpha, beta, transA, transB and the
/// C broadcast honoured as the ONNX specification states.
#[derive(Debug, Clone)]
pub struct B200Gemm {
    pub alpha: f32,
    pub beta: f32,
    pub trans_a: bool,
    pub trans_b: bool,
}

impl Default for B200Gemm {
    fn default() -> Self {
        B200Gemm { alpha: 1.0, beta: 1.0, trans_a: false, trans_b: false }
    }
}

impl B200Gemm {
    pub fn from_node(node: &Node) -> Result<Self> {
        Ok(B200Gemm {
            alpha: float(node, "alpha", 1.0),
            beta: float(node, "beta", 1.0),
            trans_a: int(node, "transA", 0) != 0,
            trans_b: int(node, "transB", 0) != 0,
        })
    }

    fn mnk(&self, a: &Shape, b: &Shape) -> Result<(usize, usize, usize)> {
        if a.len() != 2 || b.len() != 2 {
            return Err(Error::ValidationError("Gemm inputs must be 2D matrices".into()));
        }
        let (m, k) = if self.trans_a { (a[1], a[0]) } else { (a[0], a[1]) };
        let (k2, n) = if self.trans_b { (b[1], b[0]) } else { (b[0], b[1]) };
        if k != k2 {
            return Err(Error::ValidationError(format!("Incompatible dimensions for Gemm: {} vs {}", k, k2)));
        }
        Ok((m, n, k))
    }
}

impl Operator for B200Gemm {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 2, "Gemm")?;
        need_output(outputs, "Gemm")?;
        let (a, b) = (inputs[0], inputs[1]);
        let cten = inputs.get(2).copied();
        let (m, n, k) = self.mnk(&a.shape, &b.shape)?;
        let precision = precision_of(ctx)?;
        outputs[0] = with_context(ctx, |c| {
            let ad = c.upload(data_of(a)?).map_err(to_error)?;
            let bd = c.upload(data_of(b)?).map_err(to_error)?;
            let (cd, cshape) = match cten {
                Some(t) => (Some(c.upload(data_of(t)?).map_err(to_error)?), dims_i64(&t.shape)),
                None => (None, Vec::new()),
            };
            let yd = c.alloc(m * n).map_err(to_error)?;
            c.check(unsafe {
                ffi::onnxb200_gemm(c.raw(), ad.as_ptr(), bd.as_ptr(), cd.as_ref().map_or(std::ptr::null(), |t| t.as_ptr()),
                                   cshape.as_ptr(), cshape.len() as i32, m as i64, n as i64, k as i64,
                                   self.trans_a as i32, self.trans_b as i32, self.alpha, self.beta, 0, precision,
                                   yd.as_mut_ptr())
            })
            .map_err(to_error)?;
            let mut host = vec![0f32; m * n];
            yd.download(&mut host).map_err(to_error)?;
            new_tensor(vec![m, n], host)
        })?;
        Ok(())
    }

    fn output_shapes(&self, node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        let g = B200Gemm::from_node(node)?;
        let (m, n, _) = g.mnk(&known(input_shapes, 0, "Gemm")?, &known(input_shapes, 1, "Gemm")?)?;
        Ok(vec![Some(vec![m, n])])
    }

    fn validate(&self, node: &Node) -> Result<()> {
        if node.inputs.len() < 2 || node.inputs.len() > 3 {
            return Err(Error::ValidationError("Gemm requires 2 or 3 inputs".into()));
        }
        Ok(())
    }
}

// ---------------------------------------------------------------- pooling

/// MaxPool (src/ops/nn/pool.rs:168-193, :307-393) with its ONNX attributes
/// (the reference hard-codes 2x2 / stride 2, pool.rs:185-187).
#[derive(Debug, Clone, Default)]
pub struct B200MaxPool {
    pub kernel: Vec<i64>,
    pub strides: Vec<i64>,
    pub pads: Vec<i64>,
    pub ceil_mode: bool,
}

impl B200MaxPool {
    pub fn from_node(node: &Node) -> Result<Self> {
        let kernel = ints(node, "kernel_shape")
            .ok_or_else(|| Error::ValidationError("MaxPool: kernel_shape is required".into()))?;
        if kernel.len() != 2 {
            return Err(Error::UnsupportedFeature("MaxPool: only 2-D pooling is on this path".into()));
        }
        Ok(B200MaxPool {
            strides: ints(node, "strides").unwrap_or_else(|| vec![1, 1]),
            pads: ints(node, "pads").unwrap_or_else(|| vec![0, 0, 0, 0]),
            ceil_mode: int(node, "ceil_mode", 0) != 0,
            kernel,
        })
    }
}

impl Operator for B200MaxPool {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 1, "MaxPool")?;
        need_output(outputs, "MaxPool")?;
        let x = inputs[0];
        if x.shape.len() != 4 || self.kernel.len() != 2 {
            return Err(Error::UnsupportedFeature("MaxPool: only 2-D pooling is on this path".into()));
        }
        let s = dims_i64(&x.shape);
        let p = |i: usize| self.pads.get(i).copied().unwrap_or(0);
        outputs[0] = with_context(ctx, |c| {
            let xd = c.upload(data_of(x)?).map_err(to_error)?;
            // output shape first (null buffers are rejected, so run the shape
            // arithmetic of the ONNX specification here)
            let od = |i: usize, k: i64, st: i64, pb: i64, pe: i64| -> i64 {
                let span = s[i] + pb + pe - k;
                if self.ceil_mode { (span + st - 1) / st + 1 } else { span / st + 1 }
            };
            let (sh, sw) = (self.strides[0], *self.strides.get(1).unwrap_or(&self.strides[0]));
            let oh = od(2, self.kernel[0], sh, p(0), p(2));
            let ow = od(3, self.kernel[1], sw, p(1), p(3));
            let shape = vec![s[0] as usize, s[1] as usize, oh as usize, ow as usize];
            let yd = c.alloc(shape.iter().product()).map_err(to_error)?;
            let mut o = [0i64; 4];
            c.check(unsafe {
                ffi::onnxb200_maxpool2d(c.raw(), ffi::ONNXB200_LAYOUT_NCHW, s[0], s[1], s[2], s[3], self.kernel[0],
                                        self.kernel[1], sh, sw, p(0), p(1), p(2), p(3), self.ceil_mode as i32,
                                        xd.as_ptr(), yd.as_mut_ptr(), std::ptr::null_mut(), o.as_mut_ptr())
            })
            .map_err(to_error)?;
            let mut host = vec![0f32; yd.len()];
            yd.download(&mut host).map_err(to_error)?;
            new_tensor(shape, host)
        })?;
        Ok(())
    }

    fn output_shapes(&self, node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        let mp = B200MaxPool::from_node(node)?;
        let x = known(input_shapes, 0, "MaxPool")?;
        let nodes_x = vec![x[0], x[1]];
        let mut shape = nodes_x;
        for i in 0..2 {
            let st = mp.strides.get(i).copied().unwrap_or(1);
            let span = x[2 + i] as i64 + mp.pads.get(i).copied().unwrap_or(0)
                + mp.pads.get(2 + i).copied().unwrap_or(0) - mp.kernel[i];
            let o = if mp.ceil_mode { (span + st - 1) / st + 1 } else { span / st + 1 };
            shape.push(o as usize);
        }
        Ok(vec![Some(shape)])
    }

    fn validate(&self, node: &Node) -> Result<()> {
        B200MaxPool::from_node(node).map(|_| ())
    }
}

/// GlobalAveragePool (src/ops/nn/pool.rs:275-295, :493-557).
#[derive(Debug, Clone, Default)]
pub struct B200GlobalAveragePool;

impl Operator for B200GlobalAveragePool {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 1, "GlobalAveragePool")?;
        need_output(outputs, "GlobalAveragePool")?;
        let x = inputs[0];
        if x.shape.len() != 4 {
            return Err(Error::UnsupportedFeature("GlobalAveragePool: rank-4 input expected".into()));
        }
        let s = dims_i64(&x.shape);
        outputs[0] = with_context(ctx, |c| {
            let xd = c.upload(data_of(x)?).map_err(to_error)?;
            let yd = c.alloc((s[0] * s[1]) as usize).map_err(to_error)?;
            c.check(unsafe {
                ffi::onnxb200_global_avgpool(c.raw(), ffi::ONNXB200_LAYOUT_NCHW, s[0], s[1], s[2], s[3], xd.as_ptr(),
                                             yd.as_mut_ptr())
            })
            .map_err(to_error)?;
            let mut host = vec![0f32; yd.len()];
            yd.download(&mut host).map_err(to_error)?;
            new_tensor(vec![s[0] as usize, s[1] as usize, 1, 1], host)
        })?;
        Ok(())
    }

    fn output_shapes(&self, _node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        let x = known(input_shapes, 0, "GlobalAveragePool")?;
        let mut s = vec![x[0], x[1]];
        s.extend(std::iter::repeat(1).take(x.len().saturating_sub(2)));
        Ok(vec![Some(s)])
    }

    fn validate(&self, _node: &Node) -> Result<()> {
        Ok(())
    }
}

// ---------------------------------------------------------------- elementwise

/// Relu (src/ops/activations.rs:244-246): v > 0 ? v : 0 (NaN -> 0).
#[derive(Debug, Clone, Default)]
pub struct B200Relu;

impl Operator for B200Relu {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 1, "Relu")?;
        need_output(outputs, "Relu")?;
        let x = inputs[0];
        outputs[0] = with_context(ctx, |c| {
            let xd = c.upload(data_of(x)?).map_err(to_error)?;
            let yd = c.alloc(xd.len()).map_err(to_error)?;
            c.check(unsafe { ffi::onnxb200_relu(c.raw(), xd.as_ptr(), xd.len() as i64, yd.as_mut_ptr()) })
                .map_err(to_error)?;
            let mut host = vec![0f32; yd.len()];
            yd.download(&mut host).map_err(to_error)?;
            new_tensor(x.shape.clone(), host)
        })?;
        Ok(())
    }

    fn output_shapes(&self, _node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        Ok(vec![Some(known(input_shapes, 0, "Relu")?)])
    }

    fn validate(&self, _node: &Node) -> Result<()> {
        Ok(())
    }
}

/// Add with numpy broadcasting (element_wise_binary_op, src/ops/tensor.rs:1124-1218;
/// the reference registers no Add operator).
#[derive(Debug, Clone, Default)]
pub struct B200Add;

fn broadcast(a: &Shape, b: &Shape) -> Result<Shape> {
    let r = a.len().max(b.len());
    let mut o = vec![1usize; r];
    for i in 0..r {
        let da = if i >= r - a.len() { a[i - (r - a.len())] } else { 1 };
        let db = if i >= r - b.len() { b[i - (r - b.len())] } else { 1 };
        if da != db && da != 1 && db != 1 {
            return Err(Error::ValidationError(format!("Add: cannot broadcast {:?} and {:?}", a, b)));
        }
        o[i] = if da == 1 { db } else { da };
    }
    Ok(o)
}

impl Operator for B200Add {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 2, "Add")?;
        need_output(outputs, "Add")?;
        let (a, b) = (inputs[0], inputs[1]);
        let shape = broadcast(&a.shape, &b.shape)?;
        let (asz, bsz) = (dims_i64(&a.shape), dims_i64(&b.shape));
        outputs[0] = with_context(ctx, |c| {
            let ad = c.upload(data_of(a)?).map_err(to_error)?;
            let bd = c.upload(data_of(b)?).map_err(to_error)?;
            let yd = c.alloc(shape.iter().product()).map_err(to_error)?;
            c.check(unsafe {
                ffi::onnxb200_add(c.raw(), ad.as_ptr(), asz.as_ptr(), asz.len() as i32, bd.as_ptr(), bsz.as_ptr(),
                                  bsz.len() as i32, 0, yd.as_mut_ptr())
            })
            .map_err(to_error)?;
            let mut host = vec![0f32; yd.len()];
            yd.download(&mut host).map_err(to_error)?;
            new_tensor(shape.clone(), host)
        })?;
        Ok(())
    }

    fn output_shapes(&self, _node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        Ok(vec![Some(broadcast(&known(input_shapes, 0, "Add")?, &known(input_shapes, 1, "Add")?)?)])
    }

    fn validate(&self, node: &Node) -> Result<()> {
        if node.inputs.len() != 2 {
            return Err(Error::ValidationError("Add requires 2 inputs".into()));
        }
        Ok(())
    }
}

/// BatchNormalization, inference form of the ONNX specification (the reference
/// has no such operator): y = (x - mean) / sqrt(var + epsilon) * scale + B.
#[derive(Debug, Clone)]
pub struct B200BatchNormalization {
    pub epsilon: f32,
}

impl Default for B200BatchNormalization {
    fn default() -> Self {
        B200BatchNormalization { epsilon: 1e-5 }
    }
}

impl Operator for B200BatchNormalization {
    fn compute(&self, inputs: &[&Tensor], outputs: &mut [Tensor], ctx: &ExecutionContext) -> Result<()> {
        need_inputs(inputs, 5, "BatchNormalization")?;
        need_output(outputs, "BatchNormalization")?;
        let x = inputs[0];
        if x.shape.len() < 2 {
            return Err(Error::ValidationError("BatchNormalization: input rank < 2".into()));
        }
        let (n, ch) = (x.shape[0] as i64, x.shape[1] as i64);
        let spatial: usize = x.shape[2..].iter().product();
        outputs[0] = with_context(ctx, |c| {
            let xd = c.upload(data_of(x)?).map_err(to_error)?;
            let p: Vec<_> = inputs[1..5]
                .iter()
                .map(|t| c.upload(data_of(t)?).map_err(to_error))
                .collect::<Result<Vec<_>>>()?;
            let yd = c.alloc(xd.len()).map_err(to_error)?;
            c.check(unsafe {
                ffi::onnxb200_batchnorm(c.raw(), ffi::ONNXB200_LAYOUT_NCHW, n, ch, spatial as i64, 1, xd.as_ptr(),
                                        p[0].as_ptr(), p[1].as_ptr(), p[2].as_ptr(), p[3].as_ptr(), self.epsilon,
                                        yd.as_mut_ptr())
            })
            .map_err(to_error)?;
            let mut host = vec![0f32; yd.len()];
            yd.download(&mut host).map_err(to_error)?;
            new_tensor(x.shape.clone(), host)
        })?;
        Ok(())
    }

    fn output_shapes(&self, _node: &Node, input_shapes: &[Option<Shape>]) -> Result<Vec<Option<Shape>>> {
        Ok(vec![Some(known(input_shapes, 0, "BatchNormalization")?)])
    }

    fn validate(&self, node: &Node) -> Result<()> {
        if node.inputs.len() != 5 {
            return Err(Error::ValidationError("BatchNormalization requires 5 inputs".into()));
        }
        Ok(())
    }
}

// ---------------------------------------------------------------- registry

/// Registers the B200 operators under the keys the reference's standard
/// registry uses (initialize_standard_operators, src/ops/registry.rs:64-99),
/// plus Add and BatchNormalization.  Call it on a registry that does not hold
/// the CPU operators under the same keys (register_operator refuses duplicates).
pub fn register_b200_operators(registry: &mut OperatorRegistry) -> Result<()> {
    registry.register_operator("Conv", "", 11, Box::new(B200Conv::default()))?;
    registry.register_operator("MatMul", "", 9, Box::new(B200MatMul))?;
    registry.register_operator("Gemm", "", 9, Box::new(B200Gemm::default()))?;
    registry.register_operator("MaxPool", "", 11, Box::new(B200MaxPool::default()))?;
    registry.register_operator("GlobalAveragePool", "", 1, Box::new(B200GlobalAveragePool))?;
    registry.register_operator("Relu", "", 6, Box::new(B200Relu))?;
    registry.register_operator("Add", "", 7, Box::new(B200Add))?;
    registry.register_operator("BatchNormalization", "", 9, Box::new(B200BatchNormalization::default()))?;
    Ok(())
}

/// The operator instance for a node, built from the node's attributes: the
/// counterpart of OperatorRegistry::create_operator_for_node
/// (src/ops/registry.rs:101-128) for the ops of this path.
pub fn create_b200_operator_for_node(node: &Node) -> Result<Box<dyn Operator>> {
    if !node.domain.is_empty() && node.domain != "ai.onnx" {
        return Err(Error::UnsupportedFeature(format!("Operator {}.{} not supported", node.domain, node.op_type)));
    }
    Ok(match node.op_type.as_str() {
        "Conv" => Box::new(B200Conv::from_node(node)?),
        "MatMul" => Box::new(B200MatMul),
        "Gemm" => Box::new(B200Gemm::from_node(node)?),
        "MaxPool" => Box::new(B200MaxPool::from_node(node)?),
        "GlobalAveragePool" => Box::new(B200GlobalAveragePool),
        "Relu" => Box::new(B200Relu),
        "Add" => Box::new(B200Add),
        "BatchNormalization" => Box::new(B200BatchNormalization { epsilon: float(node, "epsilon", 1e-5) }),
        op => {
            return Err(Error::UnsupportedFeature(format!("Operator {}.{} not found in registry", node.domain, op)))
        }
    })
}
