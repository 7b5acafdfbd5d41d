// Graph executor: the device-side replacement of the reference's
// ExecutionEngine::prepare / run (src/execution/engine.rs:110-231) for the
// Conv / BatchNormalization / Relu / Add / MaxPool / GlobalAveragePool /
// Flatten / Gemm / MatMul path.
//
//   build:  topological order -> shape inference -> fusion (Conv + BN
//           [+ residual Add] [+ Relu]; MatMul + bias Add [+ Relu]; Gemm + Relu;
//           Add + Relu) -> NHWC layout -> weight packing into one weight arena
//           -> static memory plan of all activations in one device arena
//           (first fit, largest first, over step lifetimes; the planner's
//           optimize_memory_layout, src/memory/planner.rs:3554-3685).
//   run:    the planned steps on the handle's stream; with use_cuda_graph the
//           schedule after the input conversions is captured once into a CUDA
//           graph and replayed (the conversions run eagerly, so new input
//           pointers need no new capture, and a pipelined host run can start
//           the next batch's input copy as soon as they are done).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <new>
#include <set>
#include <string>
#include <vector>

#include "internal.h"

using namespace ob2;

namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

enum StepType {
  kInConvert,   // user NCHW -> arena NHWC (rank 4) or plain copy
  kOutConvert,  // arena -> user (NHWC -> NCHW for rank 4)
  kConv,
  kMaxPool,
  kGap,
  kAdd,
  kRelu,
  kAffine,      // standalone BatchNormalization
  kGemm,        // Gemm / MatMul with packed constant B
  kFlattenCvt,  // NHWC -> NCHW-ordered flatten when H*W > 1
};

struct GTensor {
  std::string name;
  std::vector<int64_t> shape;  // logical (NCHW for rank 4)
  bool is_init = false;
  bool is_input = false;
  bool is_output = false;
  int init_index = -1;
  size_t init_off = 0;         // offset of the device copy in the init buffer
  int cs = 0;                  // channel stride of rank-4 activations (NHWC)
  int64_t off = -1;            // arena offset
  int producer = -1;           // step index
  int last_use = -1;           // step index
  int alias_of = -1;           // Flatten view of another tensor
  bool nhwc = false;           // rank-4 image tensor stored NHWC (else row-major as given)
  bool bf16 = false;           // NHWC activation stored as bf16 (BF16 precision)
  int64_t numel() const {
    int64_t n = 1;
    for (auto v : shape) n *= v;
    return n;
  }
  size_t bytes() const {
    if (nhwc) return (size_t)shape[0] * shape[2] * shape[3] * (cs ? cs : shape[1]) * (bf16 ? 2 : 4);
    return (size_t)numel() * 4;
  }
};

struct Node {
  std::string op;
  std::vector<int> in;   // tensor ids (-1 = absent)
  std::vector<int> out;
  std::map<std::string, onnxb200_attr> attrs;
  std::map<std::string, std::vector<int64_t>> ints;
  std::map<std::string, std::string> strs;
  int64_t geti(const std::string& k, int64_t d) const {
    auto it = attrs.find(k);
    return it == attrs.end() ? d : it->second.i;
  }
  float getf(const std::string& k, float d) const {
    auto it = attrs.find(k);
    return it == attrs.end() ? d : it->second.f;
  }
  std::vector<int64_t> getv(const std::string& k, std::vector<int64_t> d) const {
    auto it = ints.find(k);
    return it == ints.end() ? d : it->second;
  }
  std::string gets(const std::string& k, const std::string& d) const {
    auto it = strs.find(k);
    return it == strs.end() ? d : it->second;
  }
};

struct Step {
  StepType type;
  std::vector<int> in;   // tensor ids read
  int out = -1;          // tensor id written
  int user_index = -1;   // graph input / output index for conversions
  int conv = -1;         // index into plans
  // pool / misc attributes
  int kh = 0, kw = 0, sh = 1, sw = 1, pt = 0, pl = 0;
  int relu = 0;
  // gemm
  int gemm = -1;
  // add: broadcast description in storage order
  int rank = 0;
  long long shape[8], sa[8], sb[8];
  long long total = 0;
  // affine
  size_t scale_off = 0, shift_off = 0;
};

struct GemmPlan {
  int M = 0, N = 0, K = 0, kpad = 0, batches = 1, prec = 0, b_rows = 0;
  size_t w_hi_off = 0, w_lo_off = 0;      // in weight arena
  size_t scale_off = SIZE_MAX, shift_off = SIZE_MAX, res_off = SIZE_MAX;  // in init buffer
  size_t aoff_off = SIZE_MAX, brow_off = SIZE_MAX;
  long long y_bstride = 0;
};

}  // namespace

struct onnxb200_graph {
  onnxb200_handle* h = nullptr;
  int device = 0;
  std::vector<GTensor> tensors;
  std::vector<Step> steps;
  std::vector<onnxb200_conv_plan> plans;
  std::vector<GemmPlan> gemms;
  std::vector<int> inputs, outputs;  // tensor ids
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  uint8_t* weights = nullptr;
  size_t weight_bytes = 0;
  uint8_t* init = nullptr;           // device copies of initializers + small tables
  size_t init_bytes = 0;
  // K-split partial sums of the steps that split (one at a time: steps run in order)
  float* split_ws = nullptr;
  size_t split_bytes = 0;
  int n_nodes_in = 0, n_fused = 0;
  int64_t kernels_per_run = -1;
  // CUDA graph state
  cudaGraph_t cg = nullptr;
  cudaGraphExec_t cge = nullptr;
  int64_t graph_kernels = 0;  // kernels inside the captured graph (all but the input conversions)
  std::vector<void*> cap_out;
  cudaStream_t cap_stream = nullptr;
  int runs = 0;
  // host-run staging
  std::vector<void*> dev_in, dev_out;
  // Recorded in every run once the input-conversion steps (run eagerly, ahead
  // of the captured graph) have read the user's input buffers: the pipelined
  // host run copies the next batch into its staging buffers after this event.
  cudaEvent_t ev_inputs_read = nullptr;
  // pipelined host run: its own copy stream and events
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t ev_copied = nullptr, ev_begin = nullptr, ev_copy_end = nullptr;
};

namespace {

int fail(onnxb200_handle* h, int code, const std::string& msg) { return set_error(h, code, msg); }

// Image tensors (rank 4, produced or consumed by image ops) live in NHWC.
bool is_rank4(const GTensor& t) { return t.nhwc; }

// Storage strides of a tensor in the iteration order used by add kernels:
// rank-4 tensors are iterated as (N, H, W, C) over their NHWC storage.
void storage_view(const GTensor& t, std::vector<int64_t>& dims, std::vector<int64_t>& strides) {
  if (is_rank4(t)) {
    const int64_t N = t.shape[0], C = t.shape[1], H = t.shape[2], W = t.shape[3];
    const int64_t cs = t.cs ? t.cs : C;
    dims = {N, H, W, C};
    strides = {H * W * cs, W * cs, cs, 1};
  } else {
    dims = t.shape;
    strides.assign(dims.size(), 0);
    int64_t e = 1;
    for (int i = (int)dims.size() - 1; i >= 0; --i) {
      strides[i] = e;
      e *= dims[i];
    }
  }
}

}  // namespace

namespace {
struct Parsed {
  std::vector<GTensor> tensors;
  std::map<std::string, int> by_name;
  std::vector<Node> nodes;
  std::vector<int> order;   // topological order of node indices
  std::vector<int> inputs;  // tensor ids of the graph inputs
  size_t init_total = 0;    // bytes of the device copies of the initializers
};
}  // namespace

// Parses the node list, orders it topologically and infers every tensor's
// shape (Operator::output_shapes per node; the planner's
// infer_node_output_shapes, src/memory/planner.rs:908-960).  Host only.
static int parse_and_infer(const onnxb200_node* nodes_in, int n_nodes, const onnxb200_tensor_info* inits,
                           int n_init, const onnxb200_tensor_info* ins, int n_inputs, bool need_data,
                           Parsed& P, std::string& msg) {
  std::map<std::string, int>& by_name = P.by_name;
  auto tensor_id = [&](const std::string& name) -> int {
    auto it = by_name.find(name);
    if (it != by_name.end()) return it->second;
    GTensor t;
    t.name = name;
    P.tensors.push_back(t);
    by_name[name] = (int)P.tensors.size() - 1;
    return (int)P.tensors.size() - 1;
  };
  auto bail = [&](int code, const std::string& m) {
    msg = m;
    return code;
  };

  // ---------------------------------------------------------------- tensors
  size_t& init_total = P.init_total;
  for (int i = 0; i < n_init; ++i) {
    if (!inits[i].name || (need_data && !inits[i].data))
      return bail(ONNXB200_ERR_INVALID_ARGUMENT, "initializer without name/data");
    if (inits[i].rank < 0 || inits[i].rank > 8 || (inits[i].rank > 0 && !inits[i].shape))
      return bail(ONNXB200_ERR_INVALID_ARGUMENT, std::string("initializer with an invalid shape: ") + inits[i].name);
    const int id = tensor_id(inits[i].name);
    GTensor& t = P.tensors[id];
    t.is_init = true;
    t.init_index = i;
    t.shape.assign(inits[i].shape, inits[i].shape + inits[i].rank);
    t.init_off = init_total;
    init_total += align_up((size_t)t.numel() * 4);
  }
  for (int i = 0; i < n_inputs; ++i) {
    if (!ins[i].name || ins[i].rank < 0 || ins[i].rank > 8 || (ins[i].rank > 0 && !ins[i].shape))
      return bail(ONNXB200_ERR_INVALID_ARGUMENT, "graph input without name / with an invalid shape");
    const int id = tensor_id(ins[i].name);
    GTensor& t = P.tensors[id];
    if (t.is_init) return bail(ONNXB200_ERR_INVALID_GRAPH, "graph input is also an initializer");
    t.is_input = true;
    t.shape.assign(ins[i].shape, ins[i].shape + ins[i].rank);
    P.inputs.push_back(id);
  }
  P.nodes.assign(n_nodes, Node());
  std::vector<Node>& nodes = P.nodes;
  for (int i = 0; i < n_nodes; ++i) {
    const onnxb200_node& src = nodes_in[i];
    Node& nd = nodes[i];
    nd.op = src.op_type ? src.op_type : "";
    if ((src.n_inputs > 0 && !src.inputs) || (src.n_outputs > 0 && !src.outputs) ||
        (src.n_attrs > 0 && !src.attrs) || src.n_inputs < 0 || src.n_outputs < 0 || src.n_attrs < 0)
      return bail(ONNXB200_ERR_INVALID_ARGUMENT, "node with null input / output / attribute arrays: " + nd.op);
    for (int j = 0; j < src.n_outputs; ++j)
      if (!src.outputs[j] || !src.outputs[j][0]) return bail(ONNXB200_ERR_INVALID_GRAPH, "node output without a name: " + nd.op);
    for (int j = 0; j < src.n_inputs; ++j) {
      const char* nm = src.inputs[j];
      nd.in.push_back((nm && nm[0]) ? tensor_id(nm) : -1);
    }
    for (int j = 0; j < src.n_outputs; ++j) nd.out.push_back(tensor_id(src.outputs[j]));
    for (int j = 0; j < src.n_attrs; ++j) {
      const onnxb200_attr& a = src.attrs[j];
      if (!a.name) continue;
      nd.attrs[a.name] = a;
      if (a.type == ONNXB200_ATTR_INTS && a.ints) nd.ints[a.name].assign(a.ints, a.ints + a.n_ints);
      if (a.type == ONNXB200_ATTR_STRING && a.s) nd.strs[a.name] = a.s;
    }
    if (nd.out.empty()) return bail(ONNXB200_ERR_INVALID_GRAPH, "node without outputs: " + nd.op);
  }

  // ---------------------------------------------------------------- topological order
  // (GraphBuilder's sort, src/parser/graph_builder.rs:12-37)
  std::vector<int> producer_node(P.tensors.size(), -1);
  for (int i = 0; i < n_nodes; ++i)
    for (int t : nodes[i].out) {
      if (producer_node[t] >= 0) return bail(ONNXB200_ERR_INVALID_GRAPH, "tensor produced twice: " + P.tensors[t].name);
      producer_node[t] = i;
    }
  std::vector<int>& order = P.order;
  {
    std::vector<int> indeg(n_nodes, 0);
    std::vector<std::vector<int>> succ(n_nodes);
    for (int i = 0; i < n_nodes; ++i)
      for (int t : nodes[i].in) {
        if (t < 0) continue;
        const GTensor& tt = P.tensors[t];
        if (producer_node[t] >= 0) {
          succ[producer_node[t]].push_back(i);
          indeg[i]++;
        } else if (!tt.is_init && !tt.is_input) {
          return bail(ONNXB200_ERR_INVALID_GRAPH, "tensor has no producer: " + tt.name);
        }
      }
    std::vector<int> ready;
    for (int i = n_nodes - 1; i >= 0; --i)
      if (indeg[i] == 0) ready.push_back(i);
    while (!ready.empty()) {
      // keep the given order among ready nodes (smallest index first)
      auto it = std::min_element(ready.begin(), ready.end());
      const int i = *it;
      ready.erase(it);
      order.push_back(i);
      for (int s : succ[i])
        if (--indeg[s] == 0) ready.push_back(s);
    }
    if ((int)order.size() != n_nodes) return bail(ONNXB200_ERR_INVALID_GRAPH, "graph has a cycle");
  }

  // ---------------------------------------------------------------- shape inference
  for (int idx : order) {
    Node& nd = nodes[idx];
    auto shp = [&](int k) -> std::vector<int64_t>& { return P.tensors[nd.in[k]].shape; };
    auto need_in = [&](int k) { return (int)nd.in.size() > k && nd.in[k] >= 0; };
    std::vector<int64_t> o;
    if (nd.op == "Conv") {
      if (!need_in(0) || !need_in(1)) return bail(ONNXB200_ERR_VALIDATION, "Conv requires at least 2 inputs");
      const auto& x = shp(0);
      const auto& w = shp(1);
      if (x.size() != 4 || w.size() != 4) return bail(ONNXB200_ERR_UNSUPPORTED, "Conv: only 2-D convolution is on this path");
      onnxb200_conv_desc d{};
      d.n = x[0]; d.c = x[1]; d.h = x[2]; d.w = x[3];
      d.c_out = w[0]; d.kh = w[2]; d.kw = w[3];
      auto st = nd.getv("strides", {1, 1});
      auto pd = nd.getv("pads", {0, 0, 0, 0});
      auto dl = nd.getv("dilations", {1, 1});
      d.stride_h = st[0]; d.stride_w = st.size() > 1 ? st[1] : st[0];
      d.pad_top = pd[0]; d.pad_left = pd.size() > 1 ? pd[1] : 0;
      d.pad_bottom = pd.size() > 2 ? pd[2] : d.pad_top; d.pad_right = pd.size() > 3 ? pd[3] : d.pad_left;
      d.dil_h = dl[0]; d.dil_w = dl.size() > 1 ? dl[1] : dl[0];
      d.group = nd.geti("group", 1);
      const std::string ap = nd.gets("auto_pad", "NOTSET");
      d.auto_pad = ap == "SAME_UPPER" ? 1 : ap == "SAME_LOWER" ? 2 : ap == "VALID" ? 3 : 0;
      if (w[1] * d.group != d.c) return bail(ONNXB200_ERR_VALIDATION, "Conv: inconsistent channel dimensions");
      int64_t shape[4];
      if (onnxb200_conv2d_output_shape(&d, shape) != ONNXB200_OK) return bail(ONNXB200_ERR_VALIDATION, "Conv: invalid attributes");
      o.assign(shape, shape + 4);
    } else if (nd.op == "BatchNormalization" || nd.op == "Relu") {
      if (!need_in(0)) return bail(ONNXB200_ERR_VALIDATION, nd.op + " requires an input");
      o = shp(0);
    } else if (nd.op == "Add") {
      if (!need_in(0) || !need_in(1)) return bail(ONNXB200_ERR_VALIDATION, "Add requires 2 inputs");
      const auto& a = shp(0);
      const auto& b = shp(1);
      const size_t r = std::max(a.size(), b.size());
      o.assign(r, 1);
      for (size_t i = 0; i < r; ++i) {
        const int64_t da = i >= r - a.size() ? a[i - (r - a.size())] : 1;
        const int64_t db = i >= r - b.size() ? b[i - (r - b.size())] : 1;
        if (da != db && da != 1 && db != 1) return bail(ONNXB200_ERR_VALIDATION, "Add: cannot broadcast shapes");
        o[i] = da == 1 ? db : da;
      }
    } else if (nd.op == "MaxPool") {
      const auto& x = shp(0);
      if (x.size() != 4) return bail(ONNXB200_ERR_UNSUPPORTED, "MaxPool: only 2-D pooling is on this path");
      auto k = nd.getv("kernel_shape", {});
      if (k.size() != 2) return bail(ONNXB200_ERR_VALIDATION, "MaxPool: kernel_shape required");
      auto st = nd.getv("strides", {1, 1});
      auto pd = nd.getv("pads", {0, 0, 0, 0});
      const int cm = (int)nd.geti("ceil_mode", 0);
      int64_t oh, ow;
      if (cm) {
        oh = (x[2] + pd[0] + pd[2] - k[0] + st[0] - 1) / st[0] + 1;
        ow = (x[3] + pd[1] + pd[3] - k[1] + st[1] - 1) / st[1] + 1;
      } else {
        oh = (x[2] + pd[0] + pd[2] - k[0]) / st[0] + 1;
        ow = (x[3] + pd[1] + pd[3] - k[1]) / st[1] + 1;
      }
      o = {x[0], x[1], oh, ow};
    } else if (nd.op == "GlobalAveragePool") {
      const auto& x = shp(0);
      if (x.size() != 4) return bail(ONNXB200_ERR_UNSUPPORTED, "GlobalAveragePool: rank-4 input expected");
      o = {x[0], x[1], 1, 1};
    } else if (nd.op == "Flatten") {
      const auto& x = shp(0);
      int64_t axis = nd.geti("axis", 1);
      if (axis < 0) axis += (int64_t)x.size();
      int64_t a = 1, b = 1;
      for (int64_t i = 0; i < (int64_t)x.size(); ++i) (i < axis ? a : b) *= x[i];
      o = {a, b};
    } else if (nd.op == "Gemm") {
      const auto& a = shp(0);
      const auto& b = shp(1);
      if (a.size() != 2 || b.size() != 2) return bail(ONNXB200_ERR_VALIDATION, "Gemm inputs must be 2D matrices");
      const int ta = (int)nd.geti("transA", 0), tb = (int)nd.geti("transB", 0);
      const int64_t m = ta ? a[1] : a[0], k1 = ta ? a[0] : a[1];
      const int64_t k2 = tb ? b[1] : b[0], n = tb ? b[0] : b[1];
      if (k1 != k2) return bail(ONNXB200_ERR_VALIDATION, "Incompatible dimensions for Gemm");
      o = {m, n};
    } else if (nd.op == "MatMul") {
      const auto& a = shp(0);
      const auto& b = shp(1);
      int64_t os[10];
      int ro = 0;
      if (onnxb200_matmul_output_shape(a.data(), (int)a.size(), b.data(), (int)b.size(), os, &ro) != ONNXB200_OK)
        return bail(ONNXB200_ERR_VALIDATION, "MatMul: incompatible shapes");
      o.assign(os, os + ro);
    } else {
      // OperatorRegistry::create_operator_for_node "not found in registry" (src/ops/registry.rs:124-127)
      return bail(ONNXB200_ERR_INVALID_OPERATOR, "operator not on this path: " + nd.op);
    }
    P.tensors[nd.out[0]].shape = o;
  }
  return ONNXB200_OK;
}

static void destroy_graph(onnxb200_graph* g) {
  if (!g) return;
  if (g->ev_inputs_read) cudaEventDestroy(g->ev_inputs_read);
  if (g->ev_copied) cudaEventDestroy(g->ev_copied);
  if (g->ev_begin) cudaEventDestroy(g->ev_begin);
  if (g->ev_copy_end) cudaEventDestroy(g->ev_copy_end);
  if (g->copy_stream) cudaStreamDestroy(g->copy_stream);
  if (g->cge) cudaGraphExecDestroy(g->cge);
  if (g->cg) cudaGraphDestroy(g->cg);
  if (g->arena) cudaFree(g->arena);
  if (g->weights) cudaFree(g->weights);
  if (g->split_ws) cudaFree(g->split_ws);
  if (g->init) cudaFree(g->init);
  for (void* p : g->dev_in) if (p) cudaFree(p);
  for (void* p : g->dev_out) if (p) cudaFree(p);
  delete g;
}

extern "C" int onnxb200_graph_destroy(onnxb200_graph* g) {
  if (!g) return ONNXB200_ERR_INVALID_ARGUMENT;
  // The graph may outlive its handle (and the handle's stream): wait on the
  // whole device instead of touching the handle.
  cudaSetDevice(g->device);
  cudaDeviceSynchronize();
  destroy_graph(g);
  return ONNXB200_OK;
}

extern "C" int onnxb200_graph_build(onnxb200_handle* h, const onnxb200_node* nodes_in, int n_nodes,
                                    const onnxb200_tensor_info* inits, int n_init,
                                    const onnxb200_tensor_info* ins, int n_inputs,
                                    const char* const* outs, int n_outputs, onnxb200_graph** out) {
  if (!h || !out || (n_nodes > 0 && !nodes_in)) return ONNXB200_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  cudaSetDevice(h->device);
  onnxb200_graph* g = new (std::nothrow) onnxb200_graph();
  if (!g) return ONNXB200_ERR_RESOURCE_EXHAUSTED;
  g->h = h;
  g->device = h->device;
  g->n_nodes_in = n_nodes;
  if (cudaEventCreateWithFlags(&g->ev_inputs_read, cudaEventDisableTiming) != cudaSuccess) {
    delete g;
    return fail(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "graph event");
  }
  Parsed P;
  std::string pmsg;
  {
    const int prc = parse_and_infer(nodes_in, n_nodes, inits, n_init, ins, n_inputs, true, P, pmsg);
    if (prc) {
      destroy_graph(g);
      return fail(h, prc, pmsg);
    }
  }
  g->tensors = std::move(P.tensors);
  g->inputs = P.inputs;
  std::map<std::string, int>& by_name = P.by_name;
  std::vector<Node>& nodes = P.nodes;
  std::vector<int>& order = P.order;
  size_t init_total = P.init_total;
  auto bail = [&](int code, const std::string& msg) {
    destroy_graph(g);
    return fail(h, code, msg);
  };
  for (int i = 0; i < n_outputs; ++i) {
    auto it = by_name.find(outs[i]);
    if (it == by_name.end()) return bail(ONNXB200_ERR_INVALID_GRAPH, std::string("unknown graph output: ") + outs[i]);
    g->tensors[it->second].is_output = true;
    g->outputs.push_back(it->second);
  }

  // ---------------------------------------------------------------- fusion
  std::vector<int> consumers(g->tensors.size(), 0);
  std::vector<std::vector<int>> consumer_nodes(g->tensors.size());
  for (int i = 0; i < n_nodes; ++i)
    for (int t : nodes[i].in)
      if (t >= 0) {
        consumers[t]++;
        consumer_nodes[t].push_back(i);
      }
  for (int t : g->outputs) consumers[t]++;
  std::vector<int> absorbed(n_nodes, 0);
  // The single consumer of `t` if it is an `op` node not yet absorbed into
  // another fused step (a residual Add has two producers that could claim it;
  // the first in topological order wins).
  auto sole_consumer = [&](int t, const char* op) -> int {
    if (consumers[t] != 1 || consumer_nodes[t].size() != 1) return -1;
    const int c = consumer_nodes[t][0];
    return (nodes[c].op == op && !absorbed[c]) ? c : -1;
  };
  auto is_const = [&](int t) { return t >= 0 && g->tensors[t].is_init; };

  struct Fused {
    int head;                 // node index of the contraction (or op)
    int last;                 // node whose position the step takes
    int bn = -1, add = -1, relu = -1;
    int residual = -1;        // tensor id
    int bias_add = -1;        // MatMul bias Add node
    int out = -1;
    int dual_head = -1, dual_bn = -1;  // a merged second 1x1 Conv + BatchNormalization
  };
  // Conv descriptor of node `ci` (NHWC, the handle's precision); epilogue not set.
  auto conv_desc_of = [&](int ci) {
    const Node& nd = nodes[ci];
    const GTensor& xt = g->tensors[nd.in[0]];
    const auto& w = g->tensors[nd.in[1]].shape;
    onnxb200_conv_desc d{};
    d.n = xt.shape[0]; d.c = xt.shape[1]; d.h = xt.shape[2]; d.w = xt.shape[3];
    d.c_out = w[0]; d.kh = w[2]; d.kw = w[3];
    auto st = nd.getv("strides", {1, 1});
    auto pd = nd.getv("pads", {0, 0, 0, 0});
    auto dl = nd.getv("dilations", {1, 1});
    d.stride_h = st[0]; d.stride_w = st.size() > 1 ? st[1] : st[0];
    d.pad_top = pd[0]; d.pad_left = pd.size() > 1 ? pd[1] : 0;
    d.pad_bottom = pd.size() > 2 ? pd[2] : d.pad_top; d.pad_right = pd.size() > 3 ? pd[3] : d.pad_left;
    d.dil_h = dl[0]; d.dil_w = dl.size() > 1 ? dl[1] : dl[0];
    d.group = nd.geti("group", 1);
    const std::string ap = nd.gets("auto_pad", "NOTSET");
    d.auto_pad = ap == "SAME_UPPER" ? 1 : ap == "SAME_LOWER" ? 2 : ap == "VALID" ? 3 : 0;
    d.layout = ONNXB200_LAYOUT_NHWC;
    d.precision = h->opts.precision;
    return d;
  };
  std::vector<Fused> fused_at(n_nodes, Fused{-1, -1});
  for (int idx : order) {
    if (absorbed[idx]) continue;
    Node& nd = nodes[idx];
    Fused f;
    f.head = idx;
    f.last = idx;
    f.out = nd.out[0];
    if (nd.op == "Conv" && is_const(nd.in[1]) && (nd.in.size() < 3 || nd.in[2] < 0 || is_const(nd.in[2]))) {
      int c = sole_consumer(f.out, "BatchNormalization");
      if (c >= 0 && !g->tensors[f.out].is_output && is_const(nodes[c].in[1]) && is_const(nodes[c].in[2]) &&
          is_const(nodes[c].in[3]) && is_const(nodes[c].in[4])) {
        f.bn = c;
        f.last = c;
        f.out = nodes[c].out[0];
        absorbed[c] = 1;
      }
      c = sole_consumer(f.out, "Add");
      if (c >= 0 && !g->tensors[f.out].is_output) {
        const int other = nodes[c].in[0] == f.out ? nodes[c].in[1] : nodes[c].in[0];
        if (other >= 0 && other != f.out && !is_const(other) && g->tensors[other].shape == g->tensors[f.out].shape) {
          f.add = c;
          f.residual = other;
          f.last = c;
          f.out = nodes[c].out[0];
          absorbed[c] = 1;
        }
      }
      c = sole_consumer(f.out, "Relu");
      if (c >= 0 && !g->tensors[f.out].is_output) {
        f.relu = c;
        f.last = c;
        f.out = nodes[c].out[0];
        absorbed[c] = 1;
      }
    } else if ((nd.op == "MatMul" || nd.op == "Gemm") && is_const(nd.in[1])) {
      if (nd.op == "MatMul") {
        const int c = sole_consumer(f.out, "Add");
        if (c >= 0 && !g->tensors[f.out].is_output) {
          const int other = nodes[c].in[0] == f.out ? nodes[c].in[1] : nodes[c].in[0];
          const auto& os = g->tensors[f.out].shape;
          if (is_const(other) && g->tensors[other].numel() == os.back() &&
              g->tensors[other].shape.back() == os.back()) {
            f.bias_add = c;
            f.last = c;
            f.out = nodes[c].out[0];
            absorbed[c] = 1;
          }
        }
      }
      const int c = sole_consumer(f.out, "Relu");
      if (c >= 0 && !g->tensors[f.out].is_output) {
        f.relu = c;
        f.last = c;
        f.out = nodes[c].out[0];
        absorbed[c] = 1;
      }
    } else if (nd.op == "Add") {
      const int c = sole_consumer(f.out, "Relu");
      if (c >= 0 && !g->tensors[f.out].is_output) {
        f.relu = c;
        f.last = c;
        f.out = nodes[c].out[0];
        absorbed[c] = 1;
      }
    }
    if (fused_at[f.last].head >= 0)
      return bail(ONNXB200_ERR_INVALID_GRAPH, "internal: two fused steps end at node " + nodes[f.last].op);
    fused_at[f.last] = f;
  }
  // Two convolutions added together -- Conv+BN -> Add(residual = Conv+BN) as in
  // a bottleneck's last 1x1 and its projection shortcut -- become one
  // two-source step when both are 1x1 convolutions the kernel can read from
  // one K loop: the shortcut's output is then never written.
  for (int idx : order) {
    Fused& f = fused_at[idx];
    if (f.head < 0 || nodes[f.head].op != "Conv" || f.bn < 0 || f.residual < 0) continue;
    const int r = f.residual;
    if (consumers[r] != 1 || g->tensors[r].is_output) continue;
    int gi = -1;
    for (int j = 0; j < n_nodes; ++j)
      if (fused_at[j].head >= 0 && fused_at[j].out == r) gi = j;
    if (gi < 0) continue;
    const Fused& gf = fused_at[gi];
    if (nodes[gf.head].op != "Conv" || gf.bn < 0 || gf.add >= 0 || gf.relu >= 0) continue;
    const Node& n1 = nodes[f.head];
    const Node& n2 = nodes[gf.head];
    if ((n1.in.size() > 2 && n1.in[2] >= 0 && !is_const(n1.in[2])) ||
        (n2.in.size() > 2 && n2.in[2] >= 0 && !is_const(n2.in[2])))
      continue;
    const onnxb200_conv_desc d1 = conv_desc_of(f.head), d2 = conv_desc_of(gf.head);
    if (g->tensors[n1.in[0]].shape.size() != 4 || g->tensors[n2.in[0]].shape.size() != 4 ||
        !dual_conv_supported(d1, (int)d1.c, d2, (int)d2.c))
      continue;
    f.dual_head = gf.head;
    f.dual_bn = gf.bn;
    f.residual = -1;
    absorbed[gf.head] = 1;
    fused_at[gi] = Fused{-1, -1};
  }
  for (int i = 0; i < n_nodes; ++i) g->n_fused += absorbed[i];

  // ---------------------------------------------------------------- layout (channel strides)
  // Rank-4 activations are images in NHWC unless a MatMul / Gemm reads or
  // writes them (those keep their row-major numpy layout).
  {
    std::vector<char> plain(g->tensors.size(), 0);
    for (int i = 0; i < n_nodes; ++i)
      if (nodes[i].op == "MatMul" || nodes[i].op == "Gemm") {
        for (int t : nodes[i].in)
          if (t >= 0) plain[t] = 1;
        for (int t : nodes[i].out) plain[t] = 1;
      }
    // elementwise ops keep the layout of their operands
    for (int i : order) {
      const Node& nd = nodes[i];
      if (nd.op != "Add" && nd.op != "Relu") continue;
      bool any_plain = false;
      for (int t : nd.in)
        if (t >= 0 && !g->tensors[t].is_init && plain[t]) any_plain = true;
      if (any_plain)
        for (int t : nd.out) plain[t] = 1;
    }
    for (int i : order) {
      const Node& nd = nodes[i];
      if (nd.op != "Add" && nd.op != "Relu") continue;
      for (int t : nd.in)
        if (t >= 0 && !g->tensors[t].is_init && g->tensors[t].shape.size() == 4 && plain[t] != plain[nd.out[0]])
          return bail(ONNXB200_ERR_UNSUPPORTED, "elementwise op mixing image and MatMul layouts: " + nd.op);
    }
    for (int i = 0; i < n_nodes; ++i) {
      const bool image_op = nodes[i].op == "Conv" || nodes[i].op == "MaxPool" ||
                            nodes[i].op == "GlobalAveragePool" || nodes[i].op == "BatchNormalization";
      if (!image_op) continue;
      for (int t : nodes[i].in)
        if (t >= 0 && plain[t] && !g->tensors[t].is_init)
          return bail(ONNXB200_ERR_UNSUPPORTED, "tensor used both as an image and as a MatMul operand: " +
                                                    g->tensors[t].name);
    }
    for (size_t t = 0; t < g->tensors.size(); ++t) {
      GTensor& tt = g->tensors[t];
      tt.nhwc = tt.shape.size() == 4 && !tt.is_init && !plain[t];
      if (tt.nhwc) tt.cs = (int)tt.shape[1];
    }
  }
  for (int id : g->inputs) {
    GTensor& t = g->tensors[id];
    if (!is_rank4(t) || t.shape[1] % 4 == 0) continue;
    bool all_conv = !consumer_nodes[id].empty();
    for (int c : consumer_nodes[id])
      if (nodes[c].op != "Conv" || nodes[c].in[0] != id || nodes[c].geti("group", 1) != 1) all_conv = false;
    if (all_conv && !t.is_output) t.cs = (int)((t.shape[1] + 3) / 4 * 4);
  }

  // ---------------------------------------------------------------- initializer upload
  g->init_bytes = init_total;
  std::vector<size_t> small_tables;  // extra regions appended to the init buffer
  size_t extra = 0;
  auto reserve_extra = [&](size_t bytes) {
    const size_t off = init_total + extra;
    extra += align_up(bytes);
    return off;
  };

  // ---------------------------------------------------------------- steps
  for (int id : g->inputs) {
    Step s;
    s.type = kInConvert;
    s.out = id;
    s.user_index = (int)(std::find(g->inputs.begin(), g->inputs.end(), id) - g->inputs.begin());
    g->steps.push_back(s);
  }
  struct PendingConv {
    int plan;
    onnxb200_conv_desc d;
    int x, w, b, bn;  // tensor ids / node
    int dual_head, dual_bn;  // second branch (nodes) of a two-source step, or -1
    int head;                // the Conv node
    int out;                 // the step's output tensor
  };
  std::vector<PendingConv> pconv;
  struct PendingGemm {
    int gp;
    int node;
    int b_id, c_id;
    int ta, tb;
    float alpha, beta;
  };
  std::vector<PendingGemm> pgemm;
  struct PendingAffine {
    size_t scale_off, shift_off;
    int bn_node;
  };
  std::vector<PendingAffine> paff;

  for (int idx : order) {
    const Fused& f = fused_at[idx];
    if (f.head < 0) continue;
    Node& nd = nodes[f.head];
    Step s;
    s.out = f.out;
    s.relu = f.relu >= 0;
    if (nd.op == "Conv") {
      const int x = nd.in[0];
      onnxb200_conv_desc d = conv_desc_of(f.head);
      const bool has_b = nd.in.size() > 2 && nd.in[2] >= 0;
      d.epilogue = (has_b ? ONNXB200_EPI_BIAS : 0) | (f.bn >= 0 ? ONNXB200_EPI_BN : 0) |
                   (f.residual >= 0 ? ONNXB200_EPI_RESIDUAL : 0) | (f.relu >= 0 ? ONNXB200_EPI_RELU : 0);
      if (f.bn >= 0) d.bn_epsilon = nodes[f.bn].getf("epsilon", 1e-5f);
      s.type = kConv;
      s.in = {x};
      if (f.residual >= 0) s.in.push_back(f.residual);
      if (f.dual_head >= 0) s.in.push_back(nodes[f.dual_head].in[0]);
      s.conv = (int)g->plans.size();
      g->plans.emplace_back();
      pconv.push_back({s.conv, d, x, nd.in[1], has_b ? nd.in[2] : -1, f.bn, f.dual_head, f.dual_bn, f.head, f.out});
    } else if (nd.op == "MaxPool") {
      auto k = nd.getv("kernel_shape", {});
      auto st = nd.getv("strides", {1, 1});
      auto pd = nd.getv("pads", {0, 0, 0, 0});
      s.type = kMaxPool;
      s.in = {nd.in[0]};
      s.kh = (int)k[0]; s.kw = (int)k[1]; s.sh = (int)st[0]; s.sw = (int)st[1];
      s.pt = (int)pd[0]; s.pl = (int)pd[1];
      if (s.relu) return bail(ONNXB200_ERR_UNSUPPORTED, "MaxPool+Relu fusion");
    } else if (nd.op == "GlobalAveragePool") {
      s.type = kGap;
      s.in = {nd.in[0]};
    } else if (nd.op == "Relu") {
      s.type = kRelu;
      s.in = {nd.in[0]};
    } else if (nd.op == "BatchNormalization") {
      for (int j = 1; j < 5; ++j)
        if (!is_const(nd.in[j])) return bail(ONNXB200_ERR_UNSUPPORTED, "BatchNormalization with non-constant parameters");
      s.type = kAffine;
      s.in = {nd.in[0]};
      s.scale_off = reserve_extra(g->tensors[nd.in[1]].numel() * 4);
      s.shift_off = reserve_extra(g->tensors[nd.in[1]].numel() * 4);
      paff.push_back({s.scale_off, s.shift_off, f.head});
    } else if (nd.op == "Add") {
      s.type = kAdd;
      s.in = {nd.in[0], nd.in[1]};
    } else if (nd.op == "Flatten") {
      const GTensor& xt = g->tensors[nd.in[0]];
      GTensor& ot = g->tensors[nd.out[0]];
      const bool view = !is_rank4(xt) || (xt.shape[2] * xt.shape[3] == 1 && xt.cs == xt.shape[1]) ||
                        nd.geti("axis", 1) == 0;
      if (view && !ot.is_output) {
        ot.alias_of = nd.in[0];
        continue;  // no step: a view of the input's storage
      }
      s.type = kFlattenCvt;
      s.in = {nd.in[0]};
    } else if (nd.op == "Gemm" || nd.op == "MatMul") {
      const int a = nd.in[0];
      const GTensor& at = g->tensors[a];
      if (!is_const(nd.in[1])) return bail(ONNXB200_ERR_UNSUPPORTED, nd.op + " with a non-constant B operand in a graph");
      if (is_rank4(at) && at.cs != at.shape[1]) return bail(ONNXB200_ERR_UNSUPPORTED, "padded MatMul input");
      GemmPlan gp;
      gp.prec = h->opts.precision == kPrecFP32 ? kPrecFP32 : h->opts.precision;
      PendingGemm pg{(int)g->gemms.size(), f.head, nd.in[1], -1, 0, 0, 1.f, 1.f};
      const auto& bs = g->tensors[nd.in[1]].shape;
      if (nd.op == "Gemm") {
        pg.ta = (int)nd.geti("transA", 0);
        pg.tb = (int)nd.geti("transB", 0);
        pg.alpha = nd.getf("alpha", 1.f);
        pg.beta = nd.getf("beta", 1.f);
        if (pg.ta) return bail(ONNXB200_ERR_UNSUPPORTED, "Gemm transA in a graph");
        gp.M = (int)at.shape[0];
        gp.K = (int)at.shape[1];
        gp.N = (int)(pg.tb ? bs[0] : bs[1]);
        if (nd.in.size() > 2 && nd.in[2] >= 0) {
          if (!is_const(nd.in[2])) return bail(ONNXB200_ERR_UNSUPPORTED, "Gemm with a non-constant C in a graph");
          pg.c_id = nd.in[2];
        }
        gp.batches = 1;
        gp.b_rows = gp.N;
      } else {
        // MatMul: A [..., M, K] activations, B [..., K, N] constant
        if (at.shape.size() < 2 || bs.size() < 2) return bail(ONNXB200_ERR_UNSUPPORTED, "1-D MatMul operand in a graph");
        gp.M = (int)at.shape[at.shape.size() - 2];
        gp.K = (int)at.shape.back();
        gp.N = (int)bs.back();
        const auto& os = g->tensors[nd.out[0]].shape;
        int64_t nbatch = 1;
        for (size_t i = 0; i + 2 < os.size(); ++i) nbatch *= os[i];
        gp.batches = (int)nbatch;
        int64_t nb_b = 1;
        for (size_t i = 0; i + 2 < bs.size(); ++i) nb_b *= bs[i];
        gp.b_rows = (int)(nb_b * gp.N);
        gp.aoff_off = reserve_extra(nbatch * sizeof(long long));
        gp.brow_off = reserve_extra(nbatch * sizeof(int));
        if (f.bias_add >= 0) {
          const Node& an = nodes[f.bias_add];
          pg.c_id = an.in[0] == nd.out[0] ? an.in[1] : an.in[0];
        }
      }
      gp.kpad = igemm_kpad(gp.K, gp.prec);
      gp.y_bstride = (long long)gp.M * gp.N;
      s.type = kGemm;
      s.in = {a};
      s.gemm = (int)g->gemms.size();
      g->gemms.push_back(gp);
      pgemm.push_back(pg);
      if (gp.K % 4 || gp.N % 4) return bail(ONNXB200_ERR_UNSUPPORTED, "Gemm/MatMul with K or N not a multiple of 4 in a graph");
    } else {
      return bail(ONNXB200_ERR_INVALID_OPERATOR, "operator not on this path: " + nd.op);
    }
    if (s.type == kAdd) {
      // broadcast in storage order
      const GTensor& A = g->tensors[s.in[0]];
      const GTensor& B = g->tensors[s.in[1]];
      const GTensor& O = g->tensors[s.out];
      std::vector<int64_t> od, os_, ad, as_, bd, bs_;
      storage_view(O, od, os_);
      const int r = (int)od.size();
      auto align_op = [&](const GTensor& t, long long* strides) {
        std::vector<int64_t> d, st;
        if (t.nhwc && O.nhwc) {
          storage_view(t, d, st);
        } else if (O.nhwc) {
          // a lower-rank constant broadcast against NHWC storage: map its NCHW
          // dims (right-aligned) onto (N, H, W, C)
          std::vector<int64_t> nchw(4, 1);
          for (size_t i = 0; i < t.shape.size(); ++i) nchw[4 - t.shape.size() + i] = t.shape[i];
          std::vector<int64_t> e(4, 0);
          int64_t acc = 1;
          for (int i = 3; i >= 0; --i) {
            e[i] = nchw[i] == 1 ? 0 : acc;
            acc *= nchw[i];
          }
          d = {nchw[0], nchw[2], nchw[3], nchw[1]};
          st = {e[0], e[2], e[3], e[1]};
        } else {
          storage_view(t, d, st);
          while ((int)d.size() < r) {
            d.insert(d.begin(), 1);
            st.insert(st.begin(), 0);
          }
        }
        for (int i = 0; i < r; ++i) strides[i] = d[i] == 1 ? 0 : st[i];
      };
      s.rank = r;
      s.total = 1;
      for (int i = 0; i < r; ++i) {
        s.shape[i] = od[i];
        s.total *= od[i];
      }
      align_op(A, s.sa);
      align_op(B, s.sb);
      if (is_rank4(O) && O.cs != O.shape[1]) return bail(ONNXB200_ERR_UNSUPPORTED, "padded Add output");
    }
    g->steps.push_back(s);
  }
  for (int i = 0; i < (int)g->outputs.size(); ++i) {
    Step s;
    s.type = kOutConvert;
    s.in = {g->outputs[i]};
    s.user_index = i;
    g->steps.push_back(s);
  }

  // ---------------------------------------------------------------- bf16 activations
  // In BF16 precision, the image tensors that convolutions (tensor cores) and
  // max pools produce are stored as bf16 when every step that reads them can:
  // a convolution reading them as its input (whole 64-channel taps) or residual,
  // a max pool (bf16 in and out), a global average pool (fp32 out).  A
  // convolution's two sources share one storage type, as do its residual and
  // output, and a bf16 input needs a bf16 output.  Graph inputs and outputs stay
  // fp32.  Decided by elimination until nothing changes.
  if (h->opts.precision == kPrecBF16) {
    std::vector<int> pc_of(g->steps.size(), -1);
    for (size_t i = 0; i < pconv.size(); ++i)
      for (size_t si = 0; si < g->steps.size(); ++si)
        if (g->steps[si].type == kConv && g->steps[si].conv == pconv[i].plan) pc_of[si] = (int)i;
    auto tc_conv = [&](int si) {
      const onnxb200_conv_desc& d = pconv[pc_of[si]].d;
      return d.group == 1 && d.c_out % 4 == 0;
    };
    for (const Step& st : g->steps) {
      if (st.out < 0) continue;
      GTensor& t = g->tensors[st.out];
      t.bf16 = t.nhwc && !t.is_input && !t.is_output && t.alias_of < 0 && t.cs == t.shape[1] &&
               t.shape[1] % 8 == 0 && ((st.type == kConv && tc_conv((int)(&st - &g->steps[0]))) ||
                                       st.type == kMaxPool);
    }
    // a view (Flatten) of a tensor is read as fp32
    for (const GTensor& t : g->tensors)
      if (t.alias_of >= 0) {
        int b = t.alias_of;
        while (g->tensors[b].alias_of >= 0) b = g->tensors[b].alias_of;
        g->tensors[b].bf16 = false;
      }
    bool changed = true;
    while (changed) {
      changed = false;
      auto off = [&](int id) {
        if (id >= 0 && g->tensors[id].bf16) {
          g->tensors[id].bf16 = false;
          changed = true;
        }
      };
      for (size_t si = 0; si < g->steps.size(); ++si) {
        const Step& st = g->steps[si];
        if (st.type == kConv) {
          const PendingConv& pc = pconv[pc_of[si]];
          const int a = st.in[0], out = st.out;
          const bool dual = pc.dual_head >= 0;
          const int res = (!dual && st.in.size() > 1) ? st.in[1] : -1;
          const int x2 = dual ? st.in[1] : -1;
          if (g->tensors[a].bf16 && (g->tensors[a].shape[1] % 64 || !tc_conv((int)si))) off(a);
          if (x2 >= 0 && g->tensors[x2].bf16 && g->tensors[x2].shape[1] % 64) off(x2);
          if (x2 >= 0 && g->tensors[a].bf16 != g->tensors[x2].bf16) { off(a); off(x2); }
          if (res >= 0 && g->tensors[res].bf16 != g->tensors[out].bf16) { off(res); off(out); }
          if (g->tensors[a].bf16 && !g->tensors[out].bf16) off(a);
        } else if (st.type == kMaxPool) {
          if (g->tensors[st.in[0]].bf16 != g->tensors[st.out].bf16) { off(st.in[0]); off(st.out); }
        } else if (st.type == kGap) {
          // reads bf16 or fp32
        } else {
          for (int t : st.in) off(t);
        }
      }
    }
  }

  // ---------------------------------------------------------------- lifetimes + arena plan
  auto base_of = [&](int t) {
    while (g->tensors[t].alias_of >= 0) t = g->tensors[t].alias_of;
    return t;
  };
  for (int si = 0; si < (int)g->steps.size(); ++si) {
    const Step& s = g->steps[si];
    if (s.out >= 0) {
      GTensor& t = g->tensors[base_of(s.out)];
      if (t.producer < 0) t.producer = si;
      t.last_use = std::max(t.last_use, si);
    }
    for (int t : s.in) {
      if (t < 0) continue;
      GTensor& tt = g->tensors[base_of(t)];
      tt.last_use = std::max(tt.last_use, si);
    }
  }
  std::vector<int> planned;
  for (int i = 0; i < (int)g->tensors.size(); ++i) {
    const GTensor& t = g->tensors[i];
    if (t.is_init || t.alias_of >= 0 || t.producer < 0) continue;
    planned.push_back(i);
  }
  std::sort(planned.begin(), planned.end(), [&](int a, int b) {
    const size_t sa = g->tensors[a].bytes(), sb = g->tensors[b].bytes();
    return sa != sb ? sa > sb : a < b;
  });
  struct Placed { size_t off, end; int first, last; };
  std::vector<Placed> placed;
  size_t arena = 0;
  for (int id : planned) {
    GTensor& t = g->tensors[id];
    const size_t sz = align_up(std::max<size_t>(t.bytes(), 4));
    // first fit among gaps left by lifetime-overlapping tensors
    std::vector<std::pair<size_t, size_t>> busy;
    for (const Placed& p : placed)
      if (!(p.last < t.producer || t.last_use < p.first)) busy.push_back({p.off, p.end});
    std::sort(busy.begin(), busy.end());
    size_t cand = 0;
    for (auto& b : busy) {
      if (cand + sz <= b.first) break;
      cand = std::max(cand, b.second);
    }
    t.off = (int64_t)cand;
    placed.push_back({cand, cand + sz, t.producer, t.last_use});
    arena = std::max(arena, cand + sz);
  }
  for (auto& t : g->tensors)
    if (t.alias_of >= 0) t.off = g->tensors[base_of(t.alias_of)].off;
  g->arena_bytes = arena;
  // every activation a step touches must have been produced and placed
  for (const Step& s : g->steps) {
    std::vector<int> ids = s.in;
    if (s.out >= 0) ids.push_back(s.out);
    for (int t : ids) {
      if (t < 0) continue;
      const GTensor& tt = g->tensors[t];
      if (!tt.is_init && tt.off < 0)
        return bail(ONNXB200_ERR_INVALID_GRAPH, "internal: tensor without storage: " + tt.name);
    }
  }

  // ---------------------------------------------------------------- device memory
  g->init_bytes = init_total + extra;
  cudaError_t e = cudaSuccess;
  if (g->arena_bytes) e = cudaMalloc(&g->arena, g->arena_bytes);
  if (e == cudaSuccess && g->init_bytes) e = cudaMalloc(&g->init, g->init_bytes);
  if (e != cudaSuccess) return bail(ONNXB200_ERR_RESOURCE_EXHAUSTED, "graph: device allocation failed");
  cudaStream_t st = h->stream;
  for (auto& t : g->tensors)
    if (t.is_init) {
      e = cudaMemcpyAsync(g->init + t.init_off, inits[t.init_index].data, (size_t)t.numel() * 4,
                          cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) return bail(ONNXB200_ERR_EXECUTION, "graph: initializer upload failed");
    }
  auto dptr = [&](int t) -> float* { return reinterpret_cast<float*>(g->init + g->tensors[t].init_off); };

  // conv plans: size, then carve from one weight arena.  scratch == nullptr:
  // size query into *used.
  auto init_plan = [&](const PendingConv& pc, void* scratch, size_t bytes, size_t* used) -> int {
    const GTensor& xt = g->tensors[pc.x];
    const int cs = xt.cs ? xt.cs : (int)xt.shape[1];
    auto branch_bn = [&](int bn_node, int conv_node) {
      ConvBranchBN b;
      const Node& bn = nodes[bn_node];
      b.scale = dptr(bn.in[1]); b.bias = dptr(bn.in[2]); b.mean = dptr(bn.in[3]); b.var = dptr(bn.in[4]);
      b.eps = bn.getf("epsilon", 1e-5f);
      const Node& cn = nodes[conv_node];
      if (cn.in.size() > 2 && cn.in[2] >= 0) b.conv_bias = dptr(cn.in[2]);
      return b;
    };
    if (pc.dual_head >= 0) {
      const Node& c2 = nodes[pc.dual_head];
      const GTensor& x2 = g->tensors[c2.in[0]];
      const onnxb200_conv_desc d2 = conv_desc_of(pc.dual_head);
      return conv_dual_plan_init(h, &pc.d, cs, dptr(pc.w), branch_bn(pc.bn, pc.head), &d2,
                                 x2.cs ? x2.cs : (int)x2.shape[1], dptr(c2.in[1]), branch_bn(pc.dual_bn, pc.dual_head),
                                 &g->plans[pc.plan], scratch, bytes, used, xt.bf16, g->tensors[pc.out].bf16);
    }
    const float *qb = pc.b >= 0 ? dptr(pc.b) : nullptr, *q1 = nullptr, *q2 = nullptr, *q3 = nullptr, *q4 = nullptr;
    if (pc.bn >= 0) {
      const Node& bn = nodes[pc.bn];
      q1 = dptr(bn.in[1]); q2 = dptr(bn.in[2]); q3 = dptr(bn.in[3]); q4 = dptr(bn.in[4]);
    }
    return conv_plan_init(h, &pc.d, cs, dptr(pc.w), qb, q1, q2, q3, q4, &g->plans[pc.plan], scratch, bytes, used,
                          xt.bf16, g->tensors[pc.out].bf16);
  };
  std::vector<size_t> plan_off(pconv.size());
  size_t wtotal = 0;
  for (size_t i = 0; i < pconv.size(); ++i) {
    const PendingConv& pc = pconv[i];
    size_t need = 0;
    int rc = init_plan(pc, nullptr, 0, &need);
    if (rc) { destroy_graph(g); return rc; }
    plan_off[i] = wtotal;
    wtotal += align_up(need);
  }
  std::vector<size_t> gemm_woff(pgemm.size());
  for (size_t i = 0; i < pgemm.size(); ++i) {
    GemmPlan& gp = g->gemms[pgemm[i].gp];
    const size_t esz = gp.prec == kPrecBF16 ? 2 : 4;
    const size_t wb = align_up((size_t)gp.b_rows * gp.kpad * esz);
    gemm_woff[i] = wtotal;
    gp.w_hi_off = wtotal;
    gp.w_lo_off = wtotal + wb;
    wtotal += wb * (gp.prec == kPrec3xTF32 ? 2 : 1);
  }
  g->weight_bytes = wtotal;
  if (wtotal) {
    e = cudaMalloc(&g->weights, wtotal);
    if (e != cudaSuccess) return bail(ONNXB200_ERR_RESOURCE_EXHAUSTED, "graph: weight allocation failed");
  }
  for (size_t i = 0; i < pconv.size(); ++i) {
    size_t used = 0;
    int rc = init_plan(pconv[i], g->weights + plan_off[i], wtotal - plan_off[i], &used);
    if (rc) { destroy_graph(g); return rc; }
  }
  // one K-split buffer for every step that splits (a few late layers and the
  // classifier at small batches; none at large ones)
  {
    size_t sb = 0;
    for (const onnxb200_conv_plan& p : g->plans)
      if (p.use_tc && p.ksplit > 1) sb = std::max(sb, p.split_bytes);
    for (const GemmPlan& gp : g->gemms)
      if (gp.batches == 1 && gp.aoff_off == SIZE_MAX && gp.brow_off == SIZE_MAX)
        sb = std::max(sb, gemm_split_bytes(h, gp.M, gp.N, gp.kpad, gp.prec, false));
    if (sb) {
      e = cudaMalloc(reinterpret_cast<void**>(&g->split_ws), sb);
      if (e != cudaSuccess) return bail(ONNXB200_ERR_RESOURCE_EXHAUSTED, "graph: K-split buffer allocation failed");
      g->split_bytes = sb;
    }
  }
  for (size_t i = 0; i < pgemm.size(); ++i) {
    const PendingGemm& pg = pgemm[i];
    GemmPlan& gp = g->gemms[pg.gp];
    const Node& nd = nodes[pg.node];
    void* hi = g->weights + gp.w_hi_off;
    void* lo = gp.prec == kPrec3xTF32 ? g->weights + gp.w_lo_off : nullptr;
    int rc;
    if (nd.op == "Gemm") {
      rc = pack_b_launch(dptr(pg.b_id), gp.N, gp.K, gp.kpad, gp.K, gp.K, gp.N, 0, pg.tb ? gp.K : 1, 0,
                         pg.tb ? 1 : gp.N, gp.prec, hi, lo, st);
    } else {
      rc = pack_b_launch(dptr(pg.b_id), gp.b_rows, gp.K, gp.kpad, gp.K, gp.K, gp.N, (long long)gp.K * gp.N, 1,
                         0, gp.N, gp.prec, hi, lo, st);
    }
    h->launches++;
    if (rc) return bail(ONNXB200_ERR_EXECUTION, "graph: weight packing failed");
    // epilogue constants: scale = alpha, shift = beta * C (row vector) or residual = beta * C
    std::vector<float> hscale, hshift;
    if (pg.alpha != 1.f) {
      hscale.assign(gp.N, pg.alpha);
      gp.scale_off = reserve_extra(gp.N * 4);
    }
    if (pg.c_id >= 0 && pg.beta != 0.f) {
      const GTensor& ct = g->tensors[pg.c_id];
      const int64_t cn = ct.shape.empty() ? 1 : ct.shape.back();
      const int64_t cm = ct.shape.size() >= 2 ? ct.shape[ct.shape.size() - 2] : 1;
      if (ct.numel() != cn * cm || (cn != 1 && cn != gp.N) || (cm != 1 && cm != gp.M))
        return bail(ONNXB200_ERR_VALIDATION, "Gemm/MatMul: C is not broadcastable");
      const float* hc = inits[ct.init_index].data;
      if (cm == 1) {
        hshift.resize(gp.N);
        for (int j = 0; j < gp.N; ++j) hshift[j] = pg.beta * hc[cn == 1 ? 0 : j];
        gp.shift_off = reserve_extra(gp.N * 4);
      } else {
        return bail(ONNXB200_ERR_UNSUPPORTED, "Gemm with a per-row C in a graph");
      }
    }
    // (re)allocate the init buffer tail for the new small tables
    if (init_total + extra > g->init_bytes) {
      uint8_t* ni = nullptr;
      e = cudaMalloc(&ni, init_total + extra);
      if (e != cudaSuccess) return bail(ONNXB200_ERR_RESOURCE_EXHAUSTED, "graph: allocation failed");
      cudaMemcpyAsync(ni, g->init, g->init_bytes, cudaMemcpyDeviceToDevice, st);
      cudaStreamSynchronize(st);
      cudaFree(g->init);
      g->init = ni;
      g->init_bytes = init_total + extra;
    }
    if (!hscale.empty()) cudaMemcpy(g->init + gp.scale_off, hscale.data(), gp.N * 4, cudaMemcpyHostToDevice);
    if (!hshift.empty()) cudaMemcpy(g->init + gp.shift_off, hshift.data(), gp.N * 4, cudaMemcpyHostToDevice);
    if (nd.op == "MatMul") {
      const auto& as = g->tensors[nd.in[0]].shape;
      const auto& bs = g->tensors[pg.b_id].shape;
      const auto& os = g->tensors[nd.out[0]].shape;
      std::vector<int64_t> ab(as.begin(), as.end() - 2), bb(bs.begin(), bs.end() - 2), ob(os.begin(), os.end() - 2);
      std::vector<long long> aoff(gp.batches);
      std::vector<int> brow(gp.batches);
      for (int b = 0; b < gp.batches; ++b) {
        int64_t ia = 0, ib = 0, sa = 1, sb = 1, rem = b;
        for (int d = (int)ob.size() - 1; d >= 0; --d) {
          const int64_t c = rem % ob[d];
          rem /= ob[d];
          const int ja = d - ((int)ob.size() - (int)ab.size());
          const int jb = d - ((int)ob.size() - (int)bb.size());
          if (ja >= 0) { if (ab[ja] != 1) ia += c * sa; sa *= ab[ja]; }
          if (jb >= 0) { if (bb[jb] != 1) ib += c * sb; sb *= bb[jb]; }
        }
        aoff[b] = ia * gp.M * gp.K;
        brow[b] = (int)(ib * gp.N);
      }
      cudaMemcpy(g->init + gp.aoff_off, aoff.data(), aoff.size() * sizeof(long long), cudaMemcpyHostToDevice);
      cudaMemcpy(g->init + gp.brow_off, brow.data(), brow.size() * sizeof(int), cudaMemcpyHostToDevice);
    }
  }
  for (const PendingAffine& pa : paff) {
    const Node& bn = nodes[pa.bn_node];
    const int C = (int)g->tensors[bn.in[1]].numel();
    int rc = bn_fold_launch(dptr(bn.in[1]), dptr(bn.in[2]), dptr(bn.in[3]), dptr(bn.in[4]), nullptr,
                            bn.getf("epsilon", 1e-5f), C, reinterpret_cast<float*>(g->init + pa.scale_off),
                            reinterpret_cast<float*>(g->init + pa.shift_off), st);
    h->launches++;
    if (rc) return bail(ONNXB200_ERR_EXECUTION, "graph: BatchNormalization fold failed");
  }
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return bail(ONNXB200_ERR_EXECUTION, std::string("graph build: ") + cudaGetErrorString(e));
  *out = g;
  return ONNXB200_OK;
}

// ---------------------------------------------------------------------------------- run
static int run_steps(onnxb200_graph* g, const float* const* uin, float* const* uout,
                     std::vector<cudaEvent_t>* ev = nullptr, size_t first = 0, size_t last = SIZE_MAX) {
  onnxb200_handle* h = g->h;
  cudaStream_t st = h->stream;
  auto T = [&](int id) -> float* {
    const GTensor& t = g->tensors[id];
    if (t.is_init) return reinterpret_cast<float*>(g->init + t.init_off);
    return reinterpret_cast<float*>(g->arena + t.off);
  };
  int rc = 0;
  last = std::min(last, g->steps.size());
  for (size_t si = first; si < last; ++si) {
    const Step& s = g->steps[si];
    if (ev) cudaEventRecord((*ev)[2 * si], st);
    switch (s.type) {
      case kInConvert: {
        const GTensor& t = g->tensors[s.out];
        if (is_rank4(t)) {
          rc = nchw_to_nhwc_launch(uin[s.user_index], (int)t.shape[0], (int)t.shape[1], (int)t.shape[2],
                                   (int)t.shape[3], t.cs, T(s.out), st);
          h->launches++;
        } else {
          rc = (int)cudaMemcpyAsync(T(s.out), uin[s.user_index], t.numel() * 4, cudaMemcpyDeviceToDevice, st);
        }
        // the input conversions come first (and are never captured): after
        // the last one the user's input buffers are free
        if (!rc && (si + 1 == g->steps.size() || g->steps[si + 1].type != kInConvert))
          rc = (int)cudaEventRecord(g->ev_inputs_read, st);
        break;
      }
      case kOutConvert: {
        const GTensor& t = g->tensors[s.in[0]];
        if (is_rank4(t) && t.shape[2] * t.shape[3] > 1) {
          rc = nhwc_to_nchw_launch(T(s.in[0]), (int)t.shape[0], (int)t.shape[1], (int)t.shape[2],
                                   (int)t.shape[3], t.cs, uout[s.user_index], st);
          h->launches++;
        } else {
          rc = (int)cudaMemcpyAsync(uout[s.user_index], T(s.in[0]), t.numel() * 4, cudaMemcpyDeviceToDevice, st);
        }
        break;
      }
      case kConv: {
        const onnxb200_conv_plan& p = g->plans[s.conv];
        if (p.dual)
          rc = conv_dual_exec_nhwc(h, &p, T(s.in[0]), T(s.in[1]), T(s.out), g->split_ws);
        else
          rc = conv_plan_exec_nhwc(h, &p, T(s.in[0]), s.in.size() > 1 ? T(s.in[1]) : nullptr, T(s.out),
                                   g->split_ws);
        if (rc) return rc;
        break;
      }
      case kMaxPool: {
        const GTensor& x = g->tensors[s.in[0]];
        const GTensor& y = g->tensors[s.out];
        if (x.bf16)
          rc = maxpool_nhwc_bf16_launch(T(s.in[0]), (int)x.shape[0], (int)x.shape[1], (int)x.shape[2],
                                        (int)x.shape[3], s.kh, s.kw, s.sh, s.sw, s.pt, s.pl, (int)y.shape[2],
                                        (int)y.shape[3], T(s.out), st);
        else
          rc = maxpool_nhwc_launch(T(s.in[0]), (int)x.shape[0], (int)x.shape[1], x.cs, (int)x.shape[2],
                                   (int)x.shape[3], s.kh, s.kw, s.sh, s.sw, s.pt, s.pl, (int)y.shape[2],
                                   (int)y.shape[3], T(s.out), nullptr, st);
        h->launches++;
        break;
      }
      case kGap: {
        const GTensor& x = g->tensors[s.in[0]];
        if (x.bf16)
          rc = gap_nhwc_bf16_launch(T(s.in[0]), (int)x.shape[0], (int)x.shape[1],
                                    (int)(x.shape[2] * x.shape[3]), T(s.out), st);
        else
          rc = gap_nhwc_launch(T(s.in[0]), (int)x.shape[0], (int)x.shape[1], (int)(x.shape[2] * x.shape[3]),
                               T(s.out), st);
        h->launches++;
        break;
      }
      case kRelu: {
        const GTensor& y = g->tensors[s.out];
        rc = relu_launch(T(s.in[0]), T(s.out), (long long)(y.bytes() / 4), st);
        h->launches++;
        break;
      }
      case kAffine: {
        const GTensor& x = g->tensors[s.in[0]];
        const float* sc = reinterpret_cast<const float*>(g->init + s.scale_off);
        const float* sh = reinterpret_cast<const float*>(g->init + s.shift_off);
        if (is_rank4(x))
          rc = channel_affine_launch(T(s.in[0]), sc, sh, T(s.out), x.shape[0] * x.shape[2] * x.shape[3],
                                     (int)x.shape[1], 1, s.relu, st);
        else {
          long long inner = 1;
          for (size_t i = 2; i < x.shape.size(); ++i) inner *= x.shape[i];
          rc = channel_affine_launch(T(s.in[0]), sc, sh, T(s.out), x.shape[0], (int)x.shape[1], inner, s.relu, st);
        }
        h->launches++;
        break;
      }
      case kAdd:
        rc = add_broadcast_launch(T(s.in[0]), T(s.in[1]), T(s.out), s.rank, s.shape, s.sa, s.sb, s.total,
                                  s.relu, st);
        h->launches++;
        break;
      case kFlattenCvt: {
        const GTensor& x = g->tensors[s.in[0]];
        rc = nhwc_to_nchw_launch(T(s.in[0]), (int)x.shape[0], (int)x.shape[1], (int)x.shape[2],
                                 (int)x.shape[3], x.cs, T(s.out), st);
        h->launches++;
        break;
      }
      case kGemm: {
        const GemmPlan& gp = g->gemms[s.gemm];
        GemmCall c;
        c.a = T(s.in[0]);
        c.M = gp.M;
        c.N = gp.N;
        c.K = gp.K;
        c.batches = gp.batches;
        c.a_off = gp.aoff_off != SIZE_MAX ? reinterpret_cast<const long long*>(g->init + gp.aoff_off) : nullptr;
        c.a_rows = (int)(g->tensors[s.in[0]].numel() / gp.K);
        c.b_row = gp.brow_off != SIZE_MAX ? reinterpret_cast<const int*>(g->init + gp.brow_off) : nullptr;
        c.y_bstride = gp.y_bstride;
        c.y = T(s.out);
        c.ldy = gp.N;
        c.scale = gp.scale_off != SIZE_MAX ? reinterpret_cast<const float*>(g->init + gp.scale_off) : nullptr;
        c.shift = gp.shift_off != SIZE_MAX ? reinterpret_cast<const float*>(g->init + gp.shift_off) : nullptr;
        c.relu = s.relu;
        if (gp.prec == kPrecFP32) {
          rc = gemm_simt_launch(c.a, reinterpret_cast<const float*>(g->weights + gp.w_hi_off), c.batches,
                                c.a_off, nullptr, c.y_bstride, c.M, c.N, c.K, c.K, gp.kpad, 0, 1, c.scale,
                                c.shift, nullptr, 0, c.relu, c.y, c.ldy, st);
          h->launches++;
          if (c.b_row) return fail(h, ONNXB200_ERR_UNSUPPORTED, "batched MatMul in fp32 CUDA-core mode");
        } else {
          c.split_ws = g->split_ws;
          c.split_bytes = g->split_bytes;
          rc = gemm_tc_run(h, c, g->weights + gp.w_hi_off,
                           gp.prec == kPrec3xTF32 ? g->weights + gp.w_lo_off : nullptr, gp.b_rows, gp.kpad,
                           gp.prec);
          if (rc) return rc;
        }
        break;
      }
    }
    if (rc) return cuda_check(h, (cudaError_t)rc, "graph step");
    if (ev) cudaEventRecord((*ev)[2 * si + 1], st);
    if (h->debug_sync) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(st, &cs);
      if (cs == cudaStreamCaptureStatusNone) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
          const int out_id = s.out >= 0 ? s.out : (s.in.empty() ? -1 : s.in[0]);
          return set_error(h, ONNXB200_ERR_EXECUTION,
                           "step " + std::to_string(si) + " (type " + std::to_string((int)s.type) +
                               ", tensor " + (out_id >= 0 ? g->tensors[out_id].name : std::string("?")) +
                               "): " + cudaGetErrorString(e));
        }
      }
    }
  }
  return ONNXB200_OK;
}

// Algorithmic work of one step: FLOPs of contractions, and bytes = every input
// read once + the output written once (fp32).
static void step_work(const onnxb200_graph* g, const Step& s, int* kind, double* flops, double* bytes) {
  // bytes as stored (channel padding and bf16 storage included)
  auto tb = [&](int id) -> double { return (double)g->tensors[id].bytes(); };
  *flops = 0;
  *bytes = 0;
  for (int t : s.in)
    if (t >= 0) *bytes += tb(t);
  if (s.out >= 0) *bytes += tb(s.out);
  switch (s.type) {
    case kInConvert:   // plus the read of the caller's NCHW fp32 buffer
      *bytes += (double)g->tensors[s.out].numel() * 4.0;
      *kind = ONNXB200_STEP_CONVERT;
      break;
    case kOutConvert:  // plus the write of the caller's fp32 buffer
      if (!s.in.empty() && s.in[0] >= 0) *bytes += (double)g->tensors[s.in[0]].numel() * 4.0;
      *kind = ONNXB200_STEP_CONVERT;
      break;
    case kFlattenCvt:
      *kind = ONNXB200_STEP_CONVERT;
      break;
    case kConv: {
      const onnxb200_conv_plan& p = g->plans[s.conv];
      const onnxb200_conv_desc& d = p.d;
      *kind = p.use_tc ? ONNXB200_STEP_CONV_TC : ONNXB200_STEP_CONV_DIRECT;
      *flops = 2.0 * d.n * p.oh * p.ow * d.c_out * (double)(d.c / d.group) * d.kh * d.kw;
      *bytes += (double)d.c_out * (d.c / d.group) * d.kh * d.kw * 4.0;
      if (p.dual) {  // the second 1x1 branch
        *flops += 2.0 * d.n * p.oh * p.ow * d.c_out * (double)p.d2.c;
        *bytes += (double)d.c_out * p.d2.c * 4.0;
      }
      break;
    }
    case kGemm: {
      const GemmPlan& gp = g->gemms[s.gemm];
      *kind = ONNXB200_STEP_GEMM;
      *flops = 2.0 * gp.batches * (double)gp.M * gp.N * gp.K;
      *bytes += (double)gp.b_rows * gp.K * 4.0;
      break;
    }
    case kMaxPool: *kind = ONNXB200_STEP_MAXPOOL; break;
    case kGap: *kind = ONNXB200_STEP_GAP; break;
    case kAdd: *kind = ONNXB200_STEP_ADD; break;
    case kRelu: *kind = ONNXB200_STEP_RELU; break;
    case kAffine: *kind = ONNXB200_STEP_AFFINE; break;
  }
}

extern "C" int onnxb200_graph_profile(onnxb200_handle* h, onnxb200_graph* g, const float* const* inputs,
                                      float* const* outputs, onnxb200_step_profile* prof, int max_steps,
                                      int* n_steps) {
  if (!h || !g || g->h != h || !n_steps) return ONNXB200_ERR_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  const size_t n = g->steps.size();
  std::vector<cudaEvent_t> ev(2 * n, nullptr);
  for (auto& e : ev)
    if (cudaEventCreate(&e) != cudaSuccess) return set_error(h, ONNXB200_ERR_EXECUTION, "profile: event");
  int rc = run_steps(g, inputs, outputs, &ev);
  if (rc == ONNXB200_OK) rc = onnxb200_synchronize(h);
  if (rc == ONNXB200_OK) {
    *n_steps = (int)n;
    for (size_t i = 0; i < n && (int)i < max_steps && prof; ++i) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1]);
      step_work(g, g->steps[i], &prof[i].kind, &prof[i].flops, &prof[i].bytes);
      prof[i].ms = ms;
    }
  }
  for (auto& e : ev) cudaEventDestroy(e);
  return rc;
}

extern "C" int onnxb200_graph_run(onnxb200_handle* h, onnxb200_graph* g, const float* const* inputs,
                                  float* const* outputs) {
  if (!h || !g || g->h != h) return ONNXB200_ERR_INVALID_ARGUMENT;
  if ((!inputs && !g->inputs.empty()) || (!outputs && !g->outputs.empty())) return ONNXB200_ERR_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  const bool use_graph = h->opts.use_cuda_graph != 0;
  std::vector<void*> vout(outputs, outputs + g->outputs.size());
  if (!use_graph || g->runs == 0) {
    // eager run (the first one also counts the kernels of one run)
    const int64_t l0 = h->launches;
    int rc = run_steps(g, inputs, outputs);
    if (rc) return rc;
    if (g->kernels_per_run < 0) g->kernels_per_run = h->launches - l0;
    g->runs++;
    return ONNXB200_OK;
  }
  // The input conversions run eagerly; the CUDA graph holds the remaining
  // steps, so it depends on the output pointers only.
  const size_t n_in = g->inputs.size();
  {
    int rc = run_steps(g, inputs, outputs, nullptr, 0, n_in);
    if (rc) return rc;
  }
  if (!g->cge || vout != g->cap_out || g->cap_stream != h->stream) {
    if (g->cge) { cudaGraphExecDestroy(g->cge); g->cge = nullptr; }
    if (g->cg) { cudaGraphDestroy(g->cg); g->cg = nullptr; }
    cudaError_t e = cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_check(h, e, "graph capture begin");
    const int64_t l0 = h->launches;
    int rc = run_steps(g, inputs, outputs, nullptr, n_in);
    g->graph_kernels = h->launches - l0;
    h->launches = l0;  // counted when replayed
    cudaGraph_t cg = nullptr;
    e = cudaStreamEndCapture(h->stream, &cg);
    if (rc) { if (cg) cudaGraphDestroy(cg); return rc; }
    if (e != cudaSuccess) return cuda_check(h, e, "graph capture end");
    e = cudaGraphInstantiate(&g->cge, cg, 0);
    if (e != cudaSuccess) { cudaGraphDestroy(cg); return cuda_check(h, e, "graph instantiate"); }
    g->cg = cg;
    g->cap_out = vout;
    g->cap_stream = h->stream;
  }
  cudaError_t e = cudaGraphLaunch(g->cge, h->stream);
  if (e != cudaSuccess) return cuda_check(h, e, "graph launch");
  h->launches += g->graph_kernels;
  g->runs++;
  return ONNXB200_OK;
}

extern "C" int onnxb200_graph_run_host(onnxb200_handle* h, onnxb200_graph* g, const float* const* inputs,
                                       float* const* outputs) {
  if (!h || !g || g->h != h) return ONNXB200_ERR_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  if (g->dev_in.empty()) {
    for (int id : g->inputs) {
      void* p = nullptr;
      if (cudaMalloc(&p, std::max<size_t>(g->tensors[id].numel() * 4, 4)) != cudaSuccess)
        return fail(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "host run: input staging allocation");
      g->dev_in.push_back(p);
    }
    for (int id : g->outputs) {
      void* p = nullptr;
      if (cudaMalloc(&p, std::max<size_t>(g->tensors[id].numel() * 4, 4)) != cudaSuccess)
        return fail(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "host run: output staging allocation");
      g->dev_out.push_back(p);
    }
  }
  for (size_t i = 0; i < g->inputs.size(); ++i) {
    cudaError_t e = cudaMemcpyAsync(g->dev_in[i], inputs[i], g->tensors[g->inputs[i]].numel() * 4,
                                    cudaMemcpyHostToDevice, h->stream);
    if (e != cudaSuccess) return cuda_check(h, e, "host run: input copy");
  }
  std::vector<const float*> din(g->dev_in.size());
  std::vector<float*> dout(g->dev_out.size());
  for (size_t i = 0; i < din.size(); ++i) din[i] = static_cast<const float*>(g->dev_in[i]);
  for (size_t i = 0; i < dout.size(); ++i) dout[i] = static_cast<float*>(g->dev_out[i]);
  int rc = onnxb200_graph_run(h, g, din.data(), dout.data());
  if (rc) return rc;
  for (size_t i = 0; i < g->outputs.size(); ++i) {
    cudaError_t e = cudaMemcpyAsync(outputs[i], g->dev_out[i], g->tensors[g->outputs[i]].numel() * 4,
                                    cudaMemcpyDeviceToHost, h->stream);
    if (e != cudaSuccess) return cuda_check(h, e, "host run: output copy");
  }
  return onnxb200_synchronize(h);
}

extern "C" int onnxb200_graph_run_host_pipelined(onnxb200_handle* h, onnxb200_graph* g, int n_batches,
                                                 const float* const* inputs, float* const* outputs) {
  if (!h || !g || g->h != h || n_batches < 0) return ONNXB200_ERR_INVALID_ARGUMENT;
  if (n_batches == 0) return ONNXB200_OK;
  if ((!inputs && !g->inputs.empty()) || (!outputs && !g->outputs.empty())) return ONNXB200_ERR_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  const size_t ni = g->inputs.size(), no = g->outputs.size();
  if (g->dev_in.empty()) {  // the same staging buffers as onnxb200_graph_run_host
    for (int id : g->inputs) {
      void* p = nullptr;
      if (cudaMalloc(&p, std::max<size_t>(g->tensors[id].numel() * 4, 4)) != cudaSuccess)
        return fail(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "host run: input staging allocation");
      g->dev_in.push_back(p);
    }
    for (int id : g->outputs) {
      void* p = nullptr;
      if (cudaMalloc(&p, std::max<size_t>(g->tensors[id].numel() * 4, 4)) != cudaSuccess)
        return fail(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "host run: output staging allocation");
      g->dev_out.push_back(p);
    }
  }
  if (!g->copy_stream) {
    if (cudaStreamCreateWithFlags(&g->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&g->ev_copied, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&g->ev_begin, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&g->ev_copy_end, cudaEventDisableTiming) != cudaSuccess)
      return fail(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "pipelined host run: stream / events");
  }
  std::vector<const float*> din(ni);
  std::vector<float*> dout(no);
  for (size_t i = 0; i < ni; ++i) din[i] = static_cast<const float*>(g->dev_in[i]);
  for (size_t i = 0; i < no; ++i) dout[i] = static_cast<float*>(g->dev_out[i]);
  cudaStream_t cs = g->copy_stream;
  // everything already queued on the handle's stream comes first
  cudaError_t e = cudaEventRecord(g->ev_begin, h->stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, g->ev_begin, 0);
  if (e != cudaSuccess) return cuda_check(h, e, "pipelined host run: ordering");
  for (int b = 0; b < n_batches; ++b) {
    // batch b's input: into the staging buffers once the previous batch's
    // graph has read them (its input-conversion steps), overlapping the rest
    // of that graph
    if (b > 0) e = cudaStreamWaitEvent(cs, g->ev_inputs_read, 0);
    for (size_t i = 0; i < ni && e == cudaSuccess; ++i)
      e = cudaMemcpyAsync(g->dev_in[i], inputs[b * ni + i], g->tensors[g->inputs[i]].numel() * 4,
                          cudaMemcpyHostToDevice, cs);
    if (e == cudaSuccess) e = cudaEventRecord(g->ev_copied, cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(h->stream, g->ev_copied, 0);
    if (e != cudaSuccess) return cuda_check(h, e, "pipelined host run: input copy");
    int rc = onnxb200_graph_run(h, g, din.data(), dout.data());
    if (rc) return rc;
    // the (small) outputs on the handle's stream, before the next batch's
    // graph rewrites the output staging buffers
    for (size_t i = 0; i < no; ++i) {
      e = cudaMemcpyAsync(outputs[b * no + i], g->dev_out[i], g->tensors[g->outputs[i]].numel() * 4,
                          cudaMemcpyDeviceToHost, h->stream);
      if (e != cudaSuccess) return cuda_check(h, e, "pipelined host run: output copy");
    }
  }
  // the handle's stream ends after the copy stream's last work
  e = cudaEventRecord(g->ev_copy_end, cs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(h->stream, g->ev_copy_end, 0);
  if (e != cudaSuccess) return cuda_check(h, e, "pipelined host run: ordering");
  return onnxb200_synchronize(h);
}

extern "C" int onnxb200_graph_output_shape(const onnxb200_graph* g, int index, int64_t* shape, int* rank) {
  if (!g || !rank || index < 0 || index >= (int)g->outputs.size()) return ONNXB200_ERR_INVALID_ARGUMENT;
  const GTensor& t = g->tensors[g->outputs[index]];
  *rank = (int)t.shape.size();
  if (shape)
    for (size_t i = 0; i < t.shape.size(); ++i) shape[i] = t.shape[i];
  return ONNXB200_OK;
}

extern "C" int onnxb200_infer_shapes(const onnxb200_node* nodes, int n_nodes, const onnxb200_tensor_info* known,
                                     int n_known, onnxb200_shape_info* shapes, int max_shapes, int* n_shapes,
                                     char* err, size_t err_len) {
  auto report = [&](int code, const std::string& m) {
    if (err && err_len) {
      std::strncpy(err, m.c_str(), err_len - 1);
      err[err_len - 1] = 0;
    }
    return code;
  };
  if (err && err_len) err[0] = 0;
  if (!n_shapes || n_nodes < 0 || n_known < 0 || (n_nodes > 0 && !nodes) || (n_known > 0 && !known) ||
      (max_shapes > 0 && !shapes))
    return report(ONNXB200_ERR_INVALID_ARGUMENT, "onnxb200_infer_shapes: null or negative argument");
  *n_shapes = 0;
  // Every known tensor is treated as an initializer: only its shape is read.
  Parsed P;
  std::string msg;
  int rc = parse_and_infer(nodes, n_nodes, known, n_known, nullptr, 0, false, P, msg);
  if (rc) return report(rc, msg);
  int n = 0;
  for (int i = 0; i < n_nodes; ++i)
    for (size_t j = 0; j < P.nodes[i].out.size(); ++j, ++n) {
      if (n >= max_shapes) continue;
      const GTensor& t = P.tensors[P.nodes[i].out[j]];
      onnxb200_shape_info& o = shapes[n];
      o.name = nodes[i].outputs[j];
      o.rank = (int)t.shape.size();
      for (int d = 0; d < 8; ++d) o.dims[d] = d < o.rank ? t.shape[d] : 0;
    }
  *n_shapes = n;
  if (n > max_shapes)
    return report(ONNXB200_ERR_RESOURCE_EXHAUSTED, "onnxb200_infer_shapes: " + std::to_string(n) +
                                                       " node outputs, room for " + std::to_string(max_shapes));
  return ONNXB200_OK;
}

extern "C" int onnxb200_graph_get_stats(const onnxb200_graph* g, onnxb200_graph_stats* s) {
  if (!g || !s) return ONNXB200_ERR_INVALID_ARGUMENT;
  s->n_nodes_in = g->n_nodes_in;
  int n = 0;
  for (const Step& st : g->steps)
    if (st.type != kInConvert && st.type != kOutConvert) n++;
  s->n_steps = n;
  s->n_fused = g->n_fused;
  s->kernels_per_run = g->kernels_per_run;
  s->arena_bytes = (int64_t)g->arena_bytes;
  s->weight_bytes = (int64_t)g->weight_bytes;
  s->captured = g->cge != nullptr;
  s->bf16_tensors = 0;
  for (const GTensor& t : g->tensors) s->bf16_tensors += t.bf16 ? 1 : 0;
  return ONNXB200_OK;
}
