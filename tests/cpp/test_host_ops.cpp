// Tests of the C++ operator interface (include/onnxb200.hpp) over libonnxb200.so.
//   test_host_ops cpu   registry, validation and shape inference (no GPU used)
//   test_host_ops gpu   compute() of every operator on small exact cases,
//                       including the reference's known answers
//                       (src/ops/nn/conv.rs:1487-1631, src/ops/math/matmul.rs:747-795)
// Prints one line per failed check and "OK <n> checks"; exit status 1 on failure.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "onnxb200.hpp"

using namespace onnxb200;

static int g_checks = 0, g_failed = 0;

#define CHECK(cond)                                                       \
  do {                                                                    \
    ++g_checks;                                                           \
    if (!(cond)) {                                                        \
      ++g_failed;                                                         \
      std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);       \
    }                                                                     \
  } while (0)

static Node node(const std::string& op, std::map<std::string, Attribute> attrs = {}) {
  Node n;
  n.op_type = op;
  n.attributes = std::move(attrs);
  return n;
}

static ShapeList shapes(std::vector<Shape> v) {
  ShapeList r;
  for (auto& s : v) r.emplace_back(s);
  return r;
}

static Shape infer(const OperatorRegistry& reg, const Node& n, std::vector<Shape> in, int* code = nullptr) {
  std::unique_ptr<Operator> op;
  Status s = reg.create_operator_for_node(n, 13, &op);
  if (!s.ok()) {
    if (code) *code = s.code;
    return {};
  }
  ShapeList out;
  s = op->output_shapes(n, shapes(std::move(in)), &out);
  if (code) *code = s.code;
  if (!s.ok() || out.empty() || !out[0]) return {};
  return *out[0];
}

static void cpu_tests() {
  OperatorRegistry reg = OperatorRegistry::initialize_standard_operators();
  // registry (registry.rs:30-128)
  CHECK(reg.get_operator("Conv", "", 11) != nullptr);
  CHECK(reg.get_operator("Conv", "", 12) == nullptr);
  CHECK(reg.register_operator("Conv", "", 11, Conv::from_node).code == ONNXB200_ERR_INVALID_OPERATOR);
  std::unique_ptr<Operator> op;
  CHECK(reg.create_operator_for_node(node("Conv"), 13, &op).ok() && std::strcmp(op->op_type(), "Conv") == 0);
  CHECK(reg.create_operator_for_node(node("Conv"), 10, &op).code == ONNXB200_ERR_UNSUPPORTED);  // only v11
  CHECK(reg.create_operator_for_node(node("Softmax"), 13, &op).code == ONNXB200_ERR_UNSUPPORTED);
  Node ai = node("Relu");
  ai.domain = "ai.onnx";
  CHECK(reg.create_operator_for_node(ai, 13, &op).ok());
  Conv conv;
  CHECK(conv.validate(node("Relu")).code == ONNXB200_ERR_VALIDATION);
  CHECK(conv.validate(node("Conv")).ok());

  // shape inference (Conv::output_shapes, conv.rs:205-323; matmul.rs:401-487; ONNX rules)
  int code = 0;
  Node stem = node("Conv", {{"strides", Attribute::of(std::vector<int64_t>{2, 2})},
                            {"pads", Attribute::of(std::vector<int64_t>{3, 3, 3, 3})}});
  CHECK((infer(reg, stem, {{1, 3, 224, 224}, {64, 3, 7, 7}}) == Shape{1, 64, 112, 112}));
  CHECK((infer(reg, node("Conv"), {{1, 1, 5}, {1, 1, 3}}) == Shape{1, 1, 3}));
  CHECK((infer(reg, node("Conv"), {{1, 1, 2, 2, 2}, {1, 1, 2, 2, 2}}) == Shape{1, 1, 1, 1, 1}));
  Node same = node("Conv", {{"auto_pad", Attribute::of(std::string("SAME_UPPER"))},
                            {"strides", Attribute::of(std::vector<int64_t>{2, 2})}});
  CHECK((infer(reg, same, {{1, 3, 9, 10}, {4, 3, 3, 3}}) == Shape{1, 4, 5, 5}));
  Node grouped = node("Conv", {{"group", Attribute::of((int64_t)3)}});
  infer(reg, grouped, {{1, 8, 5, 5}, {4, 2, 3, 3}}, &code);
  CHECK(code == ONNXB200_ERR_VALIDATION);
  CHECK((infer(reg, node("MatMul"), {{8, 1, 512, 768}, {12, 768, 3072}}) == Shape{8, 12, 512, 3072}));
  CHECK((infer(reg, node("MatMul"), {{3}, {3, 2}}) == Shape{2}));
  infer(reg, node("MatMul"), {{2, 3}, {4, 5}}, &code);
  CHECK(code == ONNXB200_ERR_VALIDATION);
  Node gemm = node("Gemm", {{"transB", Attribute::of((int64_t)1)}});
  CHECK((infer(reg, gemm, {{32, 512}, {1000, 512}}) == Shape{32, 1000}));
  Node pool = node("MaxPool", {{"kernel_shape", Attribute::of(std::vector<int64_t>{3, 3})},
                               {"strides", Attribute::of(std::vector<int64_t>{2, 2})},
                               {"pads", Attribute::of(std::vector<int64_t>{1, 1, 1, 1})}});
  CHECK((infer(reg, pool, {{2, 64, 112, 112}}) == Shape{2, 64, 56, 56}));
  CHECK((infer(reg, node("GlobalAveragePool"), {{2, 2048, 7, 7}}) == Shape{2, 2048, 1, 1}));
  CHECK((infer(reg, node("Add"), {{8, 12, 512, 3072}, {3072}}) == Shape{8, 12, 512, 3072}));
  infer(reg, node("Add"), {{2, 3}, {4}}, &code);
  CHECK(code == ONNXB200_ERR_VALIDATION);
  CHECK((infer(reg, node("Flatten"), {{2, 512, 1, 1}}) == Shape{2, 512}));
  Node flat_last = node("Flatten", {{"axis", Attribute::of((int64_t)-1)}});
  CHECK((infer(reg, flat_last, {{2, 3, 4}}) == Shape{6, 4}));
  CHECK((infer(reg, node("BatchNormalization"), {{2, 4, 5, 5}, {4}, {4}, {4}, {4}}) == Shape{2, 4, 5, 5}));
  // unknown input shapes stay unknown
  {
    std::unique_ptr<Operator> m;
    reg.create_operator_for_node(node("MatMul"), 13, &m);
    ShapeList out;
    ShapeList in{std::nullopt, Shape{3, 4}};
    CHECK(m->output_shapes(node("MatMul"), in, &out).ok() && out.size() == 1 && !out[0]);
  }
  // compute without a GPU handle is an error, not a crash
  {
    std::vector<Tensor> outs;
    Tensor x({4}, {1, -2, 3, -4});
    ExecutionContext none;
    CHECK(Relu().compute({&x}, outs, none).code == ONNXB200_ERR_INVALID_ARGUMENT);
  }
}

static bool same(const Tensor& t, const Shape& s, const std::vector<float>& v) {
  if (t.shape != s || t.data.size() != v.size()) return false;
  for (size_t i = 0; i < v.size(); ++i)
    if (t.data[i] != v[i]) {
      std::printf("  element %zu: %g != %g\n", i, t.data[i], v[i]);
      return false;
    }
  return true;
}

static std::vector<float> iota(int n, float start = 1.f) {
  std::vector<float> v(n);
  for (int i = 0; i < n; ++i) v[i] = start + i;
  return v;
}

static void gpu_tests() {
  onnxb200_handle* h = nullptr;
  CHECK(onnxb200_create(0, nullptr, &h) == ONNXB200_OK);
  if (!h) return;
  ExecutionContext ctx(h, {{"precision", "3xtf32"}});
  OperatorRegistry reg = OperatorRegistry::initialize_standard_operators();
  auto run = [&](const Node& n, std::vector<const Tensor*> in, std::vector<Tensor>* out) {
    std::unique_ptr<Operator> op;
    Status s = reg.create_operator_for_node(n, 13, &op);
    if (s.ok()) s = op->compute(in, *out, ctx);
    if (!s.ok()) std::printf("  %s: [%d] %s\n", n.op_type.c_str(), s.code, s.message.c_str());
    return s.ok();
  };
  std::vector<Tensor> out;
  {  // conv2d known answer (conv.rs:1533-1590)
    Tensor x({1, 1, 3, 3}, iota(9)), w({1, 1, 2, 2}, iota(4));
    CHECK(run(node("Conv"), {&x, &w}, &out) && same(out[0], {1, 1, 2, 2}, {37, 47, 67, 77}));
  }
  {  // conv1d known answer (conv.rs:1487-1529)
    Tensor x({1, 1, 5}, iota(5)), w({1, 1, 3}, {1, 2, 1});
    CHECK(run(node("Conv"), {&x, &w}, &out) && same(out[0], {1, 1, 3}, {8, 12, 16}));
  }
  {  // conv3d known answer (conv.rs:1594-1631)
    Tensor x({1, 1, 2, 2, 2}, iota(8)), w({1, 1, 2, 2, 2}, iota(8));
    CHECK(run(node("Conv"), {&x, &w}, &out) && same(out[0], {1, 1, 1, 1, 1}, {204}));
  }
  {  // Conv with bias, stride 2, pads
    Tensor x({1, 1, 4, 4}, iota(16)), w({1, 1, 2, 2}, {1, 0, 0, 1}), b({1}, {10});
    Node n = node("Conv", {{"strides", Attribute::of(std::vector<int64_t>{2, 2})}});
    CHECK(run(n, {&x, &w, &b}, &out) && same(out[0], {1, 1, 2, 2}, {1 + 6 + 10, 3 + 8 + 10, 9 + 14 + 10, 11 + 16 + 10}));
  }
  {  // MatMul (matmul.rs:747-795: [[1,2],[3,4]] x [[5,6],[7,8]])
    Tensor a({2, 2}, iota(4)), b({2, 2}, {5, 6, 7, 8});
    CHECK(run(node("MatMul"), {&a, &b}, &out) && same(out[0], {2, 2}, {19, 22, 43, 50}));
  }
  {  // batched broadcast MatMul: [2,1,2] x [2,2] -> [2,1,2]
    Tensor a({2, 1, 2}, {1, 2, 3, 4}), b({2, 2}, {1, 0, 0, 1});
    CHECK(run(node("MatMul"), {&a, &b}, &out) && same(out[0], {2, 1, 2}, {1, 2, 3, 4}));
  }
  {  // Gemm: alpha * A * B^T + beta * C (C broadcast over rows)
    Tensor a({2, 3}, iota(6)), b({2, 3}, {1, 0, 0, 0, 1, 0}), c({2}, {100, 200});
    Node n = node("Gemm", {{"transB", Attribute::of((int64_t)1)}, {"alpha", Attribute::of(2.f)},
                           {"beta", Attribute::of(0.5f)}});
    CHECK(run(n, {&a, &b, &c}, &out) && same(out[0], {2, 2}, {2 + 50, 4 + 100, 8 + 50, 10 + 100}));
  }
  {  // MaxPool 2x2 / 2
    Tensor x({1, 1, 4, 4}, iota(16));
    Node n = node("MaxPool", {{"kernel_shape", Attribute::of(std::vector<int64_t>{2, 2})},
                              {"strides", Attribute::of(std::vector<int64_t>{2, 2})}});
    CHECK(run(n, {&x}, &out) && same(out[0], {1, 1, 2, 2}, {6, 8, 14, 16}));
  }
  {  // GlobalAveragePool
    Tensor x({1, 2, 2, 2}, iota(8));
    CHECK(run(node("GlobalAveragePool"), {&x}, &out) && same(out[0], {1, 2, 1, 1}, {2.5f, 6.5f}));
  }
  {  // Relu
    Tensor x({4}, {1, -2, 0, -0.5f});
    CHECK(run(node("Relu"), {&x}, &out) && same(out[0], {4}, {1, 0, 0, 0}));
  }
  {  // Add with broadcasting
    Tensor a({2, 3}, iota(6)), b({3}, {10, 20, 30});
    CHECK(run(node("Add"), {&a, &b}, &out) && same(out[0], {2, 3}, {11, 22, 33, 14, 25, 36}));
  }
  {  // BatchNormalization: (x - mean) / sqrt(var + eps) * scale + bias with var + eps = 4
    Tensor x({1, 2, 1, 2}, {2, 4, 6, 8}), sc({2}, {1, 2}), bi({2}, {0, 1}), mu({2}, {0, 2}), var({2}, {4, 4});
    Node n = node("BatchNormalization", {{"epsilon", Attribute::of(0.f)}});
    CHECK(run(n, {&x, &sc, &bi, &mu, &var}, &out) && same(out[0], {1, 2, 1, 2}, {1, 2, 5, 7}));
  }
  {  // Flatten
    Tensor x({2, 2, 1, 1}, iota(4));
    CHECK(run(node("Flatten"), {&x}, &out) && same(out[0], {2, 2}, iota(4)));
  }
  {  // errors come back as statuses
    Tensor a({2, 3}, iota(6)), b({4, 5}, iota(20));
    std::unique_ptr<Operator> m;
    reg.create_operator_for_node(node("MatMul"), 13, &m);
    CHECK(m->compute({&a, &b}, out, ctx).code == ONNXB200_ERR_VALIDATION);
  }
  onnxb200_destroy(h);
}

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "cpu";
  if (mode == "cpu") cpu_tests();
  else if (mode == "gpu") gpu_tests();
  else {
    std::printf("usage: %s cpu|gpu\n", argv[0]);
    return 2;
  }
  if (g_failed) {
    std::printf("FAILED %d of %d checks\n", g_failed, g_checks);
    return 1;
  }
  std::printf("OK %d checks\n", g_checks);
  return 0;
}
