/*
 * onnxb200.hpp -- C++ host-side mirror of the onnx-rs operator interface over
 * the C ABI of onnxb200.h (header only; link libonnxb200.so).
 *
 * It keeps the reference's names, argument meanings and error behaviour so
 * that a C++ caller (or a test) reads like the reference:
 *   ExecutionContext          src/ops/registry.rs:8-11 (options) + the GPU handle
 *   Operator                  src/ops/registry.rs:14-27 (compute / input_shapes /
 *                             output_shapes / validate)
 *   OperatorRegistry          src/ops/registry.rs:30-128 (register_operator,
 *                             get_operator, initialize_standard_operators,
 *                             create_operator_for_node)
 *   Tensor                    src/ops/tensor.rs:206-218 (host fp32 data + shape)
 *   Node / Attribute          src/model.rs:162-172
 *   Status (Result<()>)       src/error.rs:19-66, codes as in onnxb200.h
 *
 * compute() takes host tensors and replaces outputs[i] wholesale with a new
 * tensor, as the reference's operators do (conv.rs:199-200): the inputs are
 * copied to the GPU, the operator runs there, the result is copied back and
 * the handle is synchronized.  Differences kept on purpose: operators are
 * configured from the node's attributes (the reference's compute() reads
 * struct defaults, conv.rs:156-203, and MaxPool hard-codes 2x2/2,
 * pool.rs:185-187); create_operator_for_node resolves the newest registered
 * version not above the model's opset (the reference compares character codes,
 * registry.rs:105-106, and never matches); BatchNormalization, Add and Flatten
 * are registered (absent from registry.rs:74-95).
 */
#ifndef ONNXB200_HPP
#define ONNXB200_HPP

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <optional>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "onnxb200.h"

namespace onnxb200 {

// ------------------------------------------------------------------ errors
// Result<()> of the reference: code 0 = Ok, otherwise an Error variant.
struct Status {
  int code = ONNXB200_OK;
  std::string message;
  bool ok() const { return code == ONNXB200_OK; }
  static Status Ok() { return {}; }
  static Status Err(int c, std::string m) { return {c, std::move(m)}; }
};

// ------------------------------------------------------------------ tensors
using Shape = std::vector<int64_t>;

inline int64_t numel_of(const Shape& s) {
  int64_t n = 1;
  for (int64_t v : s) n *= v;
  return n;
}

struct Tensor {
  std::string name;
  Shape shape;
  std::vector<float> data;  // row-major (NCHW for images)
  Tensor() = default;
  Tensor(Shape s, std::vector<float> d, std::string n = "") : name(std::move(n)), shape(std::move(s)), data(std::move(d)) {}
  static Tensor zeros(Shape s) {
    Tensor t;
    t.data.assign((size_t)numel_of(s), 0.f);
    t.shape = std::move(s);
    return t;
  }
  int64_t numel() const { return numel_of(shape); }
};

// ------------------------------------------------------------------ nodes
struct Attribute {
  enum Kind { Int, Float, Ints, String } kind = Int;
  int64_t i = 0;
  float f = 0.f;
  std::vector<int64_t> ints;
  std::string s;
  static Attribute of(int64_t v) { Attribute a; a.kind = Int; a.i = v; return a; }
  static Attribute of(float v) { Attribute a; a.kind = Float; a.f = v; return a; }
  static Attribute of(std::vector<int64_t> v) { Attribute a; a.kind = Ints; a.ints = std::move(v); return a; }
  static Attribute of(std::string v) { Attribute a; a.kind = String; a.s = std::move(v); return a; }
};

struct Node {
  std::string name, op_type, domain;
  std::vector<std::string> inputs, outputs;
  std::map<std::string, Attribute> attributes;

  int64_t get_int(const std::string& k, int64_t d) const {
    auto it = attributes.find(k);
    return it != attributes.end() && it->second.kind == Attribute::Int ? it->second.i : d;
  }
  float get_float(const std::string& k, float d) const {
    auto it = attributes.find(k);
    return it != attributes.end() && it->second.kind == Attribute::Float ? it->second.f : d;
  }
  std::vector<int64_t> get_ints(const std::string& k, std::vector<int64_t> d) const {
    auto it = attributes.find(k);
    return it != attributes.end() && it->second.kind == Attribute::Ints ? it->second.ints : d;
  }
  std::string get_string(const std::string& k, std::string d) const {
    auto it = attributes.find(k);
    return it != attributes.end() && it->second.kind == Attribute::String ? it->second.s : d;
  }
  bool has(const std::string& k) const { return attributes.count(k) != 0; }
};

// ------------------------------------------------------------------ context
// options as in the reference (e.g. "precision" = 3xtf32 | tf32 | bf16 | fp32)
// plus the GPU handle the operators run on (not owned).
class ExecutionContext {
 public:
  explicit ExecutionContext(onnxb200_handle* h = nullptr, std::map<std::string, std::string> opts = {})
      : options(std::move(opts)), handle_(h) {}
  std::map<std::string, std::string> options;
  onnxb200_handle* handle() const { return handle_; }
  int precision() const {
    auto it = options.find("precision");
    if (it == options.end()) return ONNXB200_PREC_DEFAULT;
    if (it->second == "3xtf32") return ONNXB200_PREC_3XTF32;
    if (it->second == "tf32") return ONNXB200_PREC_TF32;
    if (it->second == "bf16") return ONNXB200_PREC_BF16;
    if (it->second == "fp32") return ONNXB200_PREC_FP32;
    return ONNXB200_PREC_DEFAULT;
  }

 private:
  onnxb200_handle* handle_;
};

namespace detail {

inline Status from_code(onnxb200_handle* h, int rc, const std::string& what) {
  if (rc == ONNXB200_OK) return Status::Ok();
  const char* m = h ? onnxb200_last_error(h) : "";
  std::string msg = what + ": " + onnxb200_status_string(rc);
  if (m && *m) msg += std::string(" (") + m + ")";
  return Status::Err(rc, msg);
}

// A device copy of a host tensor (or an output buffer), freed on scope exit.
class DeviceTensor {
 public:
  DeviceTensor(onnxb200_handle* h, int64_t count) : h_(h), count_(count) {}
  DeviceTensor(const DeviceTensor&) = delete;
  DeviceTensor& operator=(const DeviceTensor&) = delete;
  ~DeviceTensor() {
    if (ptr_) onnxb200_free(h_, ptr_);
  }
  int alloc() { return onnxb200_malloc(h_, (size_t)count_ * sizeof(float), &ptr_); }
  int upload(const float* src) {
    int rc = alloc();
    if (rc) return rc;
    return onnxb200_memcpy(h_, ptr_, src, (size_t)count_ * sizeof(float), ONNXB200_COPY_H2D);
  }
  int download(float* dst) const {
    return onnxb200_memcpy(h_, dst, ptr_, (size_t)count_ * sizeof(float), ONNXB200_COPY_D2H);
  }
  float* get() const { return static_cast<float*>(ptr_); }

 private:
  onnxb200_handle* h_;
  int64_t count_;
  void* ptr_ = nullptr;
};

inline std::string shape_str(const Shape& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

}  // namespace detail

// ------------------------------------------------------------------ operator trait
using ShapeList = std::vector<std::optional<Shape>>;

class Operator {
 public:
  virtual ~Operator() = default;
  virtual const char* op_type() const = 0;
  // Replaces each outputs[i] with a new tensor (the list is resized as needed).
  virtual Status compute(const std::vector<const Tensor*>& inputs, std::vector<Tensor>& outputs,
                         const ExecutionContext& ctx) const = 0;
  virtual Status input_shapes(const Node& node, const ShapeList& in, ShapeList* out) const {
    (void)node;
    *out = in;
    return Status::Ok();
  }
  virtual Status output_shapes(const Node& node, const ShapeList& in, ShapeList* out) const = 0;
  virtual Status validate(const Node& node) const {
    if (node.op_type != op_type())
      return Status::Err(ONNXB200_ERR_VALIDATION,
                         std::string("Expected ") + op_type() + " node, got " + node.op_type);
    return Status::Ok();
  }

 protected:
  // Runs `launch` on device copies of `inputs`; output i gets out_shapes[i].
  static Status run_on_device(const std::vector<const Tensor*>& inputs, const std::vector<Shape>& out_shapes,
                              std::vector<Tensor>& outputs, const ExecutionContext& ctx, const char* what,
                              const std::function<int(const std::vector<float*>&, const std::vector<float*>&)>& launch) {
    onnxb200_handle* h = ctx.handle();
    if (!h) return Status::Err(ONNXB200_ERR_INVALID_ARGUMENT, std::string(what) + ": no GPU handle in the context");
    std::vector<std::unique_ptr<detail::DeviceTensor>> din, dout;
    std::vector<float*> pin, pout;
    for (const Tensor* t : inputs) {
      if (!t) {
        pin.push_back(nullptr);
        continue;
      }
      if ((int64_t)t->data.size() != t->numel())
        return Status::Err(ONNXB200_ERR_VALIDATION, std::string(what) + ": tensor data does not match its shape");
      din.emplace_back(new detail::DeviceTensor(h, t->numel()));
      int rc = din.back()->upload(t->data.data());
      if (rc) return detail::from_code(h, rc, what);
      pin.push_back(din.back()->get());
    }
    for (const Shape& s : out_shapes) {
      dout.emplace_back(new detail::DeviceTensor(h, numel_of(s)));
      int rc = dout.back()->alloc();
      if (rc) return detail::from_code(h, rc, what);
      pout.push_back(dout.back()->get());
    }
    int rc = launch(pin, pout);
    if (rc) return detail::from_code(h, rc, what);
    outputs.resize(out_shapes.size());
    for (size_t i = 0; i < out_shapes.size(); ++i) {
      outputs[i] = Tensor::zeros(out_shapes[i]);
      rc = dout[i]->download(outputs[i].data.data());
      if (rc) return detail::from_code(h, rc, what);
    }
    rc = onnxb200_synchronize(h);
    return detail::from_code(h, rc, what);
  }
};

// ------------------------------------------------------------------ Conv
// Conv (src/ops/nn/conv.rs:115-323): 1-D, 2-D and 3-D, with bias.
class Conv : public Operator {
 public:
  std::vector<int64_t> strides, pads, dilations;  // empty = ONNX defaults for the rank
  int64_t group = 1;
  std::string auto_pad = "NOTSET";
  static std::unique_ptr<Operator> from_node(const Node& n) {
    auto c = std::make_unique<Conv>();
    c->strides = n.get_ints("strides", {});
    c->pads = n.get_ints("pads", {});
    c->dilations = n.get_ints("dilations", {});
    c->group = n.get_int("group", 1);
    c->auto_pad = n.get_string("auto_pad", "NOTSET");
    return c;
  }
  const char* op_type() const override { return "Conv"; }

  Status desc(const Shape& x, const Shape& w, onnxb200_conv_nd_desc* d) const {
    if (x.size() < 3 || x.size() > 5 || w.size() != x.size())
      return Status::Err(ONNXB200_ERR_VALIDATION, "Conv supports only 1D, 2D, and 3D convolutions");
    const int sp = (int)x.size() - 2;
    const std::vector<int64_t> st = strides.empty() ? std::vector<int64_t>(sp, 1) : strides;
    const std::vector<int64_t> pd = pads.empty() ? std::vector<int64_t>(2 * sp, 0) : pads;
    const std::vector<int64_t> dl = dilations.empty() ? std::vector<int64_t>(sp, 1) : dilations;
    if ((int)st.size() != sp || (int)pd.size() != 2 * sp || (int)dl.size() != sp)
      return Status::Err(ONNXB200_ERR_VALIDATION, "Conv: attributes do not match the spatial rank");
    *d = onnxb200_conv_nd_desc{};
    d->spatial = sp;
    d->n = x[0];
    d->c = x[1];
    d->c_out = w[0];
    d->group = group;
    for (int i = 0; i < sp; ++i) {
      d->in[i] = x[2 + i];
      d->kernel[i] = w[2 + i];
      d->stride[i] = st[i];
      d->pad_begin[i] = pd[i];
      d->pad_end[i] = pd[sp + i];
      d->dilation[i] = dl[i];
    }
    d->auto_pad = auto_pad == "SAME_UPPER"   ? ONNXB200_AUTOPAD_SAME_UPPER
                  : auto_pad == "SAME_LOWER" ? ONNXB200_AUTOPAD_SAME_LOWER
                  : auto_pad == "VALID"      ? ONNXB200_AUTOPAD_VALID
                                             : ONNXB200_AUTOPAD_NOTSET;
    if (w[1] * (group > 0 ? group : 1) != x[1])
      return Status::Err(ONNXB200_ERR_VALIDATION, "Conv: inconsistent channel dimensions");
    return Status::Ok();
  }
  Status output_shape(const Shape& x, const Shape& w, Shape* out) const {
    onnxb200_conv_nd_desc d;
    Status s = desc(x, w, &d);
    if (!s.ok()) return s;
    int64_t o[5];
    int rank = 0;
    int rc = onnxb200_conv_nd_output_shape(&d, o, &rank);
    if (rc) return Status::Err(rc, "Conv: invalid shapes or attributes");
    out->assign(o, o + rank);
    return Status::Ok();
  }
  Status output_shapes(const Node& node, const ShapeList& in, ShapeList* out) const override {
    if (in.size() < 2)
      return Status::Err(ONNXB200_ERR_VALIDATION, "Conv requires at least 2 inputs, got " + std::to_string(in.size()));
    out->assign(1, std::nullopt);
    if (!in[0] || !in[1]) return Status::Ok();
    auto c = from_node(node);
    Shape o;
    Status s = static_cast<Conv*>(c.get())->output_shape(*in[0], *in[1], &o);
    if (s.ok()) (*out)[0] = o;
    return s;
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.size() < 2 || !in[0] || !in[1]) return Status::Err(ONNXB200_ERR_VALIDATION, "Conv requires X and W");
    onnxb200_conv_nd_desc d;
    Status s = desc(in[0]->shape, in[1]->shape, &d);
    if (!s.ok()) return s;
    Shape o;
    s = output_shape(in[0]->shape, in[1]->shape, &o);
    if (!s.ok()) return s;
    const bool has_b = in.size() > 2 && in[2];
    const int prec = ctx.precision();
    return run_on_device(in, {o}, outputs, ctx, "Conv", [&](const std::vector<float*>& x, const std::vector<float*>& y) {
      if (d.spatial != 2) return onnxb200_conv_nd(ctx.handle(), &d, x[0], x[1], has_b ? x[2] : nullptr, y[0]);
      onnxb200_conv_desc c{};
      c.n = d.n; c.c = d.c; c.h = d.in[0]; c.w = d.in[1];
      c.c_out = d.c_out; c.kh = d.kernel[0]; c.kw = d.kernel[1];
      c.stride_h = d.stride[0]; c.stride_w = d.stride[1];
      c.pad_top = d.pad_begin[0]; c.pad_left = d.pad_begin[1];
      c.pad_bottom = d.pad_end[0]; c.pad_right = d.pad_end[1];
      c.dil_h = d.dilation[0]; c.dil_w = d.dilation[1];
      c.group = d.group;
      c.auto_pad = d.auto_pad;
      c.layout = ONNXB200_LAYOUT_NCHW;
      c.epilogue = has_b ? ONNXB200_EPI_BIAS : 0;
      c.precision = prec;
      return onnxb200_conv2d(ctx.handle(), &c, x[0], x[1], has_b ? x[2] : nullptr, nullptr, nullptr, nullptr,
                             nullptr, nullptr, y[0]);
    });
  }
};

// ------------------------------------------------------------------ MatMul / Gemm
// MatMul (src/ops/math/matmul.rs:60-124): numpy-broadcast batched matmul.
class MatMul : public Operator {
 public:
  static std::unique_ptr<Operator> from_node(const Node&) { return std::make_unique<MatMul>(); }
  const char* op_type() const override { return "MatMul"; }
  static Status output_shape(const Shape& a, const Shape& b, Shape* out) {
    int64_t o[16];
    int r = 0;
    if (a.size() > 15 || b.size() > 15) return Status::Err(ONNXB200_ERR_VALIDATION, "MatMul: rank too large");
    int rc = onnxb200_matmul_output_shape(a.data(), (int)a.size(), b.data(), (int)b.size(), o, &r);
    if (rc)
      return Status::Err(rc, "Incompatible shapes for MatMul: " + detail::shape_str(a) + " and " + detail::shape_str(b));
    out->assign(o, o + r);
    return Status::Ok();
  }
  Status output_shapes(const Node&, const ShapeList& in, ShapeList* out) const override {
    if (in.size() < 2) return Status::Err(ONNXB200_ERR_VALIDATION, "MatMul requires 2 inputs");
    out->assign(1, std::nullopt);
    if (!in[0] || !in[1]) return Status::Ok();
    Shape o;
    Status s = output_shape(*in[0], *in[1], &o);
    if (s.ok()) (*out)[0] = o;
    return s;
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.size() < 2 || !in[0] || !in[1]) return Status::Err(ONNXB200_ERR_VALIDATION, "MatMul requires 2 inputs");
    Shape o;
    Status s = output_shape(in[0]->shape, in[1]->shape, &o);
    if (!s.ok()) return s;
    const Shape& as = in[0]->shape;
    const Shape& bs = in[1]->shape;
    const int prec = ctx.precision();
    return run_on_device({in[0], in[1]}, {o}, outputs, ctx, "MatMul",
                         [&](const std::vector<float*>& x, const std::vector<float*>& y) {
                           return onnxb200_matmul(ctx.handle(), x[0], as.data(), (int)as.size(), x[1], bs.data(),
                                                  (int)bs.size(), nullptr, 0, prec, y[0]);
                         });
  }
};

// Gemm (src/ops/math/gemm.rs:17-44) with alpha, beta, transA, transB honoured.
class Gemm : public Operator {
 public:
  float alpha = 1.f, beta = 1.f;
  int64_t trans_a = 0, trans_b = 0;
  static std::unique_ptr<Operator> from_node(const Node& n) {
    auto g = std::make_unique<Gemm>();
    g->alpha = n.get_float("alpha", 1.f);
    g->beta = n.get_float("beta", 1.f);
    g->trans_a = n.get_int("transA", 0);
    g->trans_b = n.get_int("transB", 0);
    return g;
  }
  const char* op_type() const override { return "Gemm"; }
  Status dims(const Shape& a, const Shape& b, int64_t* m, int64_t* n, int64_t* k) const {
    if (a.size() != 2 || b.size() != 2) return Status::Err(ONNXB200_ERR_VALIDATION, "Gemm inputs must be 2D matrices");
    *m = trans_a ? a[1] : a[0];
    *k = trans_a ? a[0] : a[1];
    const int64_t k2 = trans_b ? b[1] : b[0];
    *n = trans_b ? b[0] : b[1];
    if (*k != k2)
      return Status::Err(ONNXB200_ERR_VALIDATION,
                         "Incompatible dimensions for Gemm: " + std::to_string(*k) + " and " + std::to_string(k2));
    return Status::Ok();
  }
  Status output_shapes(const Node& node, const ShapeList& in, ShapeList* out) const override {
    if (in.size() < 2) return Status::Err(ONNXB200_ERR_VALIDATION, "Gemm requires at least 2 inputs");
    out->assign(1, std::nullopt);
    if (!in[0] || !in[1]) return Status::Ok();
    auto g = from_node(node);
    int64_t m, n, k;
    Status s = static_cast<Gemm*>(g.get())->dims(*in[0], *in[1], &m, &n, &k);
    if (s.ok()) (*out)[0] = Shape{m, n};
    return s;
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.size() < 2 || !in[0] || !in[1]) return Status::Err(ONNXB200_ERR_VALIDATION, "Gemm requires A and B");
    int64_t m, n, k;
    Status s = dims(in[0]->shape, in[1]->shape, &m, &n, &k);
    if (!s.ok()) return s;
    const Tensor* c = in.size() > 2 ? in[2] : nullptr;
    const Shape cs = c ? c->shape : Shape{1};
    const int prec = ctx.precision();
    return run_on_device({in[0], in[1], c}, {{m, n}}, outputs, ctx, "Gemm",
                         [&](const std::vector<float*>& x, const std::vector<float*>& y) {
                           return onnxb200_gemm(ctx.handle(), x[0], x[1], x[2], cs.data(), c ? (int)cs.size() : 0, m, n,
                                                k, (int)trans_a, (int)trans_b, alpha, beta, 0, prec, y[0]);
                         });
  }
};

// ------------------------------------------------------------------ pooling
// MaxPool (src/ops/nn/pool.rs:168-193) with the node's attributes.
class MaxPool : public Operator {
 public:
  std::vector<int64_t> kernel_shape{2, 2}, strides{1, 1}, pads{0, 0, 0, 0};
  int64_t ceil_mode = 0;
  static std::unique_ptr<Operator> from_node(const Node& n) {
    auto p = std::make_unique<MaxPool>();
    p->kernel_shape = n.get_ints("kernel_shape", {2, 2});
    p->strides = n.get_ints("strides", {1, 1});
    p->pads = n.get_ints("pads", {0, 0, 0, 0});
    p->ceil_mode = n.get_int("ceil_mode", 0);
    return p;
  }
  const char* op_type() const override { return "MaxPool"; }
  Status out_shape(const Shape& x, Shape* o) const {
    if (x.size() != 4 || kernel_shape.size() != 2 || strides.size() != 2 || pads.size() != 4)
      return Status::Err(ONNXB200_ERR_UNSUPPORTED, "MaxPool: 2-D pooling of NCHW input only");
    int64_t hw[2];
    for (int i = 0; i < 2; ++i) {
      const int64_t span = x[2 + i] + pads[i] + pads[2 + i] - kernel_shape[i];
      if (span < 0 || strides[i] <= 0) return Status::Err(ONNXB200_ERR_VALIDATION, "MaxPool: window larger than input");
      hw[i] = (ceil_mode ? (span + strides[i] - 1) / strides[i] : span / strides[i]) + 1;
    }
    *o = Shape{x[0], x[1], hw[0], hw[1]};
    return Status::Ok();
  }
  Status output_shapes(const Node& node, const ShapeList& in, ShapeList* out) const override {
    out->assign(1, std::nullopt);
    if (in.empty() || !in[0]) return Status::Ok();
    auto p = from_node(node);
    Shape o;
    Status s = static_cast<MaxPool*>(p.get())->out_shape(*in[0], &o);
    if (s.ok()) (*out)[0] = o;
    return s;
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.empty() || !in[0]) return Status::Err(ONNXB200_ERR_VALIDATION, "MaxPool requires an input");
    Shape o;
    Status s = out_shape(in[0]->shape, &o);
    if (!s.ok()) return s;
    const Shape& x = in[0]->shape;
    return run_on_device({in[0]}, {o}, outputs, ctx, "MaxPool", [&](const std::vector<float*>& xi, const std::vector<float*>& y) {
      int64_t out4[4];
      return onnxb200_maxpool2d(ctx.handle(), ONNXB200_LAYOUT_NCHW, x[0], x[1], x[2], x[3], kernel_shape[0],
                                kernel_shape[1], strides[0], strides[1], pads[0], pads[1], pads[2], pads[3],
                                (int)ceil_mode, xi[0], y[0], nullptr, out4);
    });
  }
};

// GlobalAveragePool (src/ops/nn/pool.rs:275-295 -> global_pool :493-557).
class GlobalAveragePool : public Operator {
 public:
  static std::unique_ptr<Operator> from_node(const Node&) { return std::make_unique<GlobalAveragePool>(); }
  const char* op_type() const override { return "GlobalAveragePool"; }
  Status output_shapes(const Node&, const ShapeList& in, ShapeList* out) const override {
    out->assign(1, std::nullopt);
    if (in.empty() || !in[0]) return Status::Ok();
    Shape o{(*in[0])[0], (*in[0])[1]};
    for (size_t i = 2; i < in[0]->size(); ++i) o.push_back(1);
    (*out)[0] = o;
    return Status::Ok();
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.empty() || !in[0] || in[0]->shape.size() != 4)
      return Status::Err(ONNXB200_ERR_VALIDATION, "GlobalAveragePool requires an NCHW input");
    const Shape& x = in[0]->shape;
    return run_on_device({in[0]}, {{x[0], x[1], 1, 1}}, outputs, ctx, "GlobalAveragePool",
                         [&](const std::vector<float*>& xi, const std::vector<float*>& y) {
                           return onnxb200_global_avgpool(ctx.handle(), ONNXB200_LAYOUT_NCHW, x[0], x[1], x[2], x[3],
                                                          xi[0], y[0]);
                         });
  }
};

// ------------------------------------------------------------------ elementwise
// Relu (src/ops/activations.rs:92-96, relu :244-246).
class Relu : public Operator {
 public:
  static std::unique_ptr<Operator> from_node(const Node&) { return std::make_unique<Relu>(); }
  const char* op_type() const override { return "Relu"; }
  Status output_shapes(const Node&, const ShapeList& in, ShapeList* out) const override {
    out->assign(1, in.empty() ? std::nullopt : in[0]);
    return Status::Ok();
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.empty() || !in[0]) return Status::Err(ONNXB200_ERR_VALIDATION, "Relu requires an input");
    const int64_t n = in[0]->numel();
    return run_on_device({in[0]}, {in[0]->shape}, outputs, ctx, "Relu",
                         [&](const std::vector<float*>& x, const std::vector<float*>& y) {
                           return onnxb200_relu(ctx.handle(), x[0], n, y[0]);
                         });
  }
};

// Add = element_wise_binary_op(+) with broadcasting (src/ops/tensor.rs:1124-1218).
class Add : public Operator {
 public:
  static std::unique_ptr<Operator> from_node(const Node&) { return std::make_unique<Add>(); }
  const char* op_type() const override { return "Add"; }
  // get_broadcast_shape (src/ops/tensor.rs:1536-1571)
  static Status broadcast(const Shape& a, const Shape& b, Shape* out) {
    const size_t r = a.size() > b.size() ? a.size() : b.size();
    out->assign(r, 1);
    for (size_t i = 0; i < r; ++i) {
      const int64_t x = i + a.size() >= r ? a[i + a.size() - r] : 1;
      const int64_t y = i + b.size() >= r ? b[i + b.size() - r] : 1;
      if (x != y && x != 1 && y != 1)
        return Status::Err(ONNXB200_ERR_VALIDATION, "Cannot broadcast shapes " + detail::shape_str(a) + " and " +
                                                        detail::shape_str(b) + ": incompatible dimensions at index " +
                                                        std::to_string(i));
      (*out)[i] = x == 1 ? y : x;
    }
    return Status::Ok();
  }
  Status output_shapes(const Node&, const ShapeList& in, ShapeList* out) const override {
    if (in.size() < 2) return Status::Err(ONNXB200_ERR_VALIDATION, "Add requires 2 inputs");
    out->assign(1, std::nullopt);
    if (!in[0] || !in[1]) return Status::Ok();
    Shape o;
    Status s = broadcast(*in[0], *in[1], &o);
    if (s.ok()) (*out)[0] = o;
    return s;
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.size() < 2 || !in[0] || !in[1]) return Status::Err(ONNXB200_ERR_VALIDATION, "Add requires 2 inputs");
    Shape o;
    Status s = broadcast(in[0]->shape, in[1]->shape, &o);
    if (!s.ok()) return s;
    const Shape& as = in[0]->shape;
    const Shape& bs = in[1]->shape;
    return run_on_device({in[0], in[1]}, {o}, outputs, ctx, "Add",
                         [&](const std::vector<float*>& x, const std::vector<float*>& y) {
                           return onnxb200_add(ctx.handle(), x[0], as.data(), (int)as.size(), x[1], bs.data(),
                                               (int)bs.size(), 0, y[0]);
                         });
  }
};

// ONNX BatchNormalization (inference); not in the reference registry.
class BatchNormalization : public Operator {
 public:
  float epsilon = 1e-5f;
  static std::unique_ptr<Operator> from_node(const Node& n) {
    auto b = std::make_unique<BatchNormalization>();
    b->epsilon = n.get_float("epsilon", 1e-5f);
    return b;
  }
  const char* op_type() const override { return "BatchNormalization"; }
  Status output_shapes(const Node&, const ShapeList& in, ShapeList* out) const override {
    out->assign(1, in.empty() ? std::nullopt : in[0]);
    return Status::Ok();
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext& ctx) const override {
    if (in.size() < 5) return Status::Err(ONNXB200_ERR_VALIDATION, "BatchNormalization requires 5 inputs");
    for (int i = 0; i < 5; ++i)
      if (!in[i]) return Status::Err(ONNXB200_ERR_VALIDATION, "BatchNormalization requires 5 inputs");
    const Shape& x = in[0]->shape;
    if (x.size() != 4) return Status::Err(ONNXB200_ERR_UNSUPPORTED, "BatchNormalization: NCHW input only");
    return run_on_device({in[0], in[1], in[2], in[3], in[4]}, {x}, outputs, ctx, "BatchNormalization",
                         [&](const std::vector<float*>& p, const std::vector<float*>& y) {
                           return onnxb200_batchnorm(ctx.handle(), ONNXB200_LAYOUT_NCHW, x[0], x[1], x[2], x[3], p[0],
                                                     p[1], p[2], p[3], p[4], epsilon, y[0]);
                         });
  }
};

// ONNX Flatten (a view; the reference only infers its shape, src/memory/planner.rs:1735).
class Flatten : public Operator {
 public:
  int64_t axis = 1;
  static std::unique_ptr<Operator> from_node(const Node& n) {
    auto f = std::make_unique<Flatten>();
    f->axis = n.get_int("axis", 1);
    return f;
  }
  const char* op_type() const override { return "Flatten"; }
  Status out_shape(const Shape& x, Shape* o) const {
    const int64_t r = (int64_t)x.size();
    const int64_t ax = axis < 0 ? axis + r : axis;
    if (ax < 0 || ax > r) return Status::Err(ONNXB200_ERR_VALIDATION, "Flatten: axis out of range");
    int64_t a = 1, b = 1;
    for (int64_t i = 0; i < r; ++i) (i < ax ? a : b) *= x[i];
    *o = Shape{a, b};
    return Status::Ok();
  }
  Status output_shapes(const Node& node, const ShapeList& in, ShapeList* out) const override {
    out->assign(1, std::nullopt);
    if (in.empty() || !in[0]) return Status::Ok();
    auto f = from_node(node);
    Shape o;
    Status s = static_cast<Flatten*>(f.get())->out_shape(*in[0], &o);
    if (s.ok()) (*out)[0] = o;
    return s;
  }
  Status compute(const std::vector<const Tensor*>& in, std::vector<Tensor>& outputs,
                 const ExecutionContext&) const override {
    if (in.empty() || !in[0]) return Status::Err(ONNXB200_ERR_VALIDATION, "Flatten requires an input");
    Shape o;
    Status s = out_shape(in[0]->shape, &o);
    if (!s.ok()) return s;
    outputs.resize(1);
    outputs[0] = Tensor(o, in[0]->data);
    return Status::Ok();
  }
};

// ------------------------------------------------------------------ registry
class OperatorRegistry {
 public:
  using Factory = std::function<std::unique_ptr<Operator>(const Node&)>;

  Status register_operator(const std::string& name, const std::string& domain, int64_t version, Factory f) {
    const auto key = std::make_tuple(name, domain, version);
    if (operators_.count(key))
      return Status::Err(ONNXB200_ERR_INVALID_OPERATOR, "Operator " + domain + "." + name + " (version " +
                                                            std::to_string(version) + ") is already registered");
    operators_[key] = std::move(f);
    return Status::Ok();
  }
  // The registered factory, or nullptr.
  const Factory* get_operator(const std::string& name, const std::string& domain, int64_t version) const {
    auto it = operators_.find(std::make_tuple(name, domain, version));
    return it == operators_.end() ? nullptr : &it->second;
  }
  // Versions as registered by the reference (registry.rs:74-95); BN, Add and
  // Flatten are additions for this path.
  static OperatorRegistry initialize_standard_operators() {
    OperatorRegistry r;
    r.register_operator("MatMul", "", 9, MatMul::from_node);
    r.register_operator("Gemm", "", 9, Gemm::from_node);
    r.register_operator("Conv", "", 11, Conv::from_node);
    r.register_operator("MaxPool", "", 11, MaxPool::from_node);
    r.register_operator("GlobalAveragePool", "", 1, GlobalAveragePool::from_node);
    r.register_operator("Relu", "", 6, Relu::from_node);
    r.register_operator("Add", "", 7, Add::from_node);
    r.register_operator("BatchNormalization", "", 9, BatchNormalization::from_node);
    r.register_operator("Flatten", "", 9, Flatten::from_node);
    return r;
  }
  // The newest registered version <= opset_version, configured from the node.
  Status create_operator_for_node(const Node& node, int64_t opset_version, std::unique_ptr<Operator>* out) const {
    const std::string domain = node.domain == "ai.onnx" ? "" : node.domain;
    const Factory* best = nullptr;
    int64_t best_v = -1;
    for (const auto& kv : operators_) {
      if (std::get<0>(kv.first) == node.op_type && std::get<1>(kv.first) == domain &&
          std::get<2>(kv.first) <= opset_version && std::get<2>(kv.first) > best_v) {
        best = &kv.second;
        best_v = std::get<2>(kv.first);
      }
    }
    if (!best)
      return Status::Err(ONNXB200_ERR_UNSUPPORTED,
                         "Operator " + domain + "." + node.op_type + " not found in registry");
    *out = (*best)(node);
    return (*out)->validate(node);
  }

 private:
  std::map<std::tuple<std::string, std::string, int64_t>, Factory> operators_;
};

}  // namespace onnxb200

#endif  // ONNXB200_HPP
