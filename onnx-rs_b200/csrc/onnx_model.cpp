// ONNX ModelProto reader: the protobuf wire format decoded by hand (no
// protobuf library), restricted to what the Conv / MatMul / Gemm path needs --
// the main graph's nodes and attributes, its fp32 initializers (inline or in
// an external data file), its inputs and outputs with shapes, and the opset
// imports -- and handed to onnxb200_graph_build.
//
// Follows OnnxModelLoader (src/parser/model_loader.rs:27-454):
//   load_model / load_model_from_bytes (:27-43), convert_proto_to_internal
//   (:51-89; a model without a graph is an error), handle_opset_imports
//   (:190-203; the default domain starts at version 1), convert_graph_proto
//   (:205-256), convert_node_proto (:325-344), convert_tensor_proto (:346-451;
//   raw_data first, else the typed repeated field), convert_value_info_proto /
//   extract_type_info (:453-531; dim_param -> -1, a value without a type is an
//   error), convert_attribute_proto (:534-660; type UNDEFINED is an error).
// Field numbers are those of proto/onnx.proto:65-470, which are the standard
// ONNX numbers, except for TensorProto fields 13 / 14: real .onnx files store
// external data as repeated key/value entries (field 13) plus a data_location
// enum (field 14), and that is what is read here.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <new>
#include <set>
#include <string>
#include <vector>

#include "internal.h"

namespace {

// --------------------------------------------------------------- wire format
enum WireType { kVarint = 0, kFixed64 = 1, kLen = 2, kFixed32 = 5 };

struct ParseError {
  int code;
  std::string msg;
};

[[noreturn]] void raise(int code, const std::string& msg) { throw ParseError{code, msg}; }

struct Field {
  uint32_t num = 0;
  int wire = 0;
  uint64_t v = 0;              // varint / fixed value
  const uint8_t* data = nullptr;  // length-delimited payload
  size_t len = 0;
};

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  Cursor(const uint8_t* b, size_t n) : p(b), end(b + n) {}
  bool done() const { return p >= end; }

  uint64_t varint() {
    uint64_t r = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p >= end) raise(ONNXB200_ERR_PROTOBUF, "truncated varint");
      const uint8_t b = *p++;
      r |= (uint64_t)(b & 0x7f) << shift;
      if (!(b & 0x80)) return r;
    }
    raise(ONNXB200_ERR_PROTOBUF, "varint longer than 10 bytes");
  }
  uint64_t fixed(int bytes) {
    if ((size_t)(end - p) < (size_t)bytes) raise(ONNXB200_ERR_PROTOBUF, "truncated fixed-width field");
    uint64_t r = 0;
    for (int i = 0; i < bytes; ++i) r |= (uint64_t)p[i] << (8 * i);
    p += bytes;
    return r;
  }
  Field next() {
    Field f;
    const uint64_t key = varint();
    f.num = (uint32_t)(key >> 3);
    f.wire = (int)(key & 7);
    if (f.num == 0) raise(ONNXB200_ERR_PROTOBUF, "field number 0");
    switch (f.wire) {
      case kVarint: f.v = varint(); break;
      case kFixed64: f.v = fixed(8); break;
      case kFixed32: f.v = fixed(4); break;
      case kLen: {
        const uint64_t n = varint();
        if (n > (uint64_t)(end - p)) raise(ONNXB200_ERR_PROTOBUF, "length-delimited field runs past its message");
        f.data = p;
        f.len = (size_t)n;
        p += n;
        break;
      }
      default: raise(ONNXB200_ERR_PROTOBUF, "unsupported wire type " + std::to_string(f.wire));
    }
    return f;
  }
};

std::string str(const Field& f) {
  if (f.wire != kLen) raise(ONNXB200_ERR_PROTOBUF, "string field with wire type " + std::to_string(f.wire));
  return std::string(reinterpret_cast<const char*>(f.data), f.len);
}
int64_t i64(const Field& f) {
  if (f.wire != kVarint) raise(ONNXB200_ERR_PROTOBUF, "integer field with wire type " + std::to_string(f.wire));
  return (int64_t)f.v;
}
float f32(const Field& f) {
  if (f.wire != kFixed32) raise(ONNXB200_ERR_PROTOBUF, "float field with wire type " + std::to_string(f.wire));
  const uint32_t u = (uint32_t)f.v;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}
// repeated int64: packed (one length-delimited run) or one varint per entry
void rep_i64(const Field& f, std::vector<int64_t>& out) {
  if (f.wire == kVarint) { out.push_back((int64_t)f.v); return; }
  if (f.wire != kLen) raise(ONNXB200_ERR_PROTOBUF, "repeated integer field with wire type " + std::to_string(f.wire));
  Cursor c(f.data, f.len);
  while (!c.done()) out.push_back((int64_t)c.varint());
}
// repeated float: packed or one fixed32 per entry
void rep_f32(const Field& f, std::vector<float>& out) {
  if (f.wire == kFixed32) { out.push_back(f32(f)); return; }
  if (f.wire != kLen || f.len % 4) raise(ONNXB200_ERR_PROTOBUF, "malformed repeated float field");
  const size_t n0 = out.size();
  out.resize(n0 + f.len / 4);
  std::memcpy(out.data() + n0, f.data, f.len);  // little-endian host
}

// --------------------------------------------------------------- model
constexpr int kFloat = 1;  // TensorProto.DataType.FLOAT (proto/onnx.proto:241)

struct MAttr {
  std::string name;
  int type = -1;  // ONNXB200_ATTR_*
  int64_t i = 0;
  float f = 0.f;
  std::vector<int64_t> ints;
  std::string s;
};
struct MNode {
  std::string name, op, domain;
  std::vector<std::string> in, out;
  std::vector<MAttr> attrs;
};
struct MTensor {
  std::string name;
  int dtype = 0;
  std::vector<int64_t> dims;
  std::vector<float> data;
  bool have_data = false;
  bool external = false;
  std::string location;
  int64_t offset = 0, length = -1;
};
struct MValue {
  std::string name;
  int elem = 0;
  std::vector<int64_t> dims;
};

int64_t numel(const std::vector<int64_t>& d) {
  int64_t n = 1;
  for (int64_t v : d) {
    if (v < 0 || (v > 0 && n > INT64_MAX / v)) raise(ONNXB200_ERR_INVALID_MODEL, "bad tensor dimension");
    n *= v;
  }
  return n;
}

// TensorShapeProto.Dimension (proto/onnx.proto:444-455): dim_value, or -1 for dim_param
void parse_shape(const Field& sf, std::vector<int64_t>& dims) {
  Cursor c(sf.data, sf.len);
  while (!c.done()) {
    Field f = c.next();
    if (f.num != 1 || f.wire != kLen) continue;
    Cursor d(f.data, f.len);
    bool have = false;
    int64_t v = -1;
    while (!d.done()) {
      Field g = d.next();
      if (g.num == 1) { v = i64(g); have = true; }
      else if (g.num == 2) { v = -1; have = true; }
    }
    if (!have) raise(ONNXB200_ERR_INVALID_MODEL, "tensor shape dimension without dim_value or dim_param");
    dims.push_back(v);
  }
}

// ValueInfoProto (proto/onnx.proto:365-374) with TypeProto.Tensor (:379-385)
MValue parse_value_info(const Field& vf) {
  MValue v;
  bool have_type = false;
  Cursor c(vf.data, vf.len);
  while (!c.done()) {
    Field f = c.next();
    if (f.num == 1) v.name = str(f);
    else if (f.num == 2 && f.wire == kLen) {
      have_type = true;
      Cursor t(f.data, f.len);
      while (!t.done()) {
        Field g = t.next();
        if ((g.num == 1 || g.num == 8) && g.wire == kLen) {  // tensor_type / sparse_tensor_type
          Cursor tt(g.data, g.len);
          while (!tt.done()) {
            Field h = tt.next();
            if (h.num == 1) v.elem = (int)i64(h);
            else if (h.num == 2 && h.wire == kLen) parse_shape(h, v.dims);
          }
        } else if (g.num == 4 || g.num == 5) {  // sequence / map: 1-D of unknown size
          v.dims = {-1};
        }
      }
    }
  }
  if (!have_type) raise(ONNXB200_ERR_INVALID_MODEL, "missing type for value info: " + v.name);
  return v;
}

// TensorProto (proto/onnx.proto:235-339)
MTensor parse_tensor(const Field& tf) {
  MTensor t;
  std::vector<float> fdata;
  const uint8_t* raw = nullptr;
  size_t raw_len = 0;
  bool have_raw = false, segment = false;
  int location = 0;
  std::vector<std::pair<std::string, std::string>> ext;
  Cursor c(tf.data, tf.len);
  while (!c.done()) {
    Field f = c.next();
    switch (f.num) {
      case 1: rep_i64(f, t.dims); break;
      case 2: t.dtype = (int)i64(f); break;
      case 3: segment = true; break;
      case 4: rep_f32(f, fdata); break;
      case 8: t.name = str(f); break;
      case 9:
        if (f.wire != kLen) raise(ONNXB200_ERR_PROTOBUF, "raw_data with wire type " + std::to_string(f.wire));
        raw = f.data;
        raw_len = f.len;
        have_raw = true;
        break;
      case 13: {  // StringStringEntryProto {key = 1, value = 2}
        if (f.wire != kLen) raise(ONNXB200_ERR_PROTOBUF, "external_data entry with wire type " + std::to_string(f.wire));
        Cursor e(f.data, f.len);
        std::string k, v;
        while (!e.done()) {
          Field g = e.next();
          if (g.num == 1) k = str(g);
          else if (g.num == 2) v = str(g);
        }
        ext.emplace_back(k, v);
        break;
      }
      case 14: location = (int)i64(f); break;
      default: break;  // int32/int64/double/uint64/string data, doc_string: not fp32
    }
  }
  if (t.dtype != kFloat) return t;  // kept as metadata only
  if (segment) raise(ONNXB200_ERR_UNSUPPORTED, "segmented tensor " + t.name);
  const int64_t n = numel(t.dims);
  if (location == 1) {
    t.external = true;
    for (auto& kv : ext) {
      char* endp = nullptr;
      if (kv.first == "location") t.location = kv.second;
      else if (kv.first == "offset") t.offset = std::strtoll(kv.second.c_str(), &endp, 10);
      else if (kv.first == "length") t.length = std::strtoll(kv.second.c_str(), &endp, 10);
    }
    if (t.location.empty()) raise(ONNXB200_ERR_INVALID_MODEL, "external tensor " + t.name + " without a location");
    if (t.length >= 0 && t.length != n * 4)
      raise(ONNXB200_ERR_INVALID_MODEL, "external tensor " + t.name + ": length does not match its shape");
    return t;
  }
  if (have_raw) {
    if ((int64_t)raw_len != n * 4)
      raise(ONNXB200_ERR_INVALID_MODEL, "tensor " + t.name + ": raw_data size does not match its shape");
    t.data.resize((size_t)n);
    if (n) std::memcpy(t.data.data(), raw, raw_len);  // little-endian host
  } else {
    if ((int64_t)fdata.size() != n)
      raise(ONNXB200_ERR_INVALID_MODEL, "tensor " + t.name + ": float_data size does not match its shape");
    t.data.swap(fdata);
  }
  t.have_data = true;
  return t;
}

// AttributeProto (proto/onnx.proto:175-231); types with no onnxb200_attr form
// (tensors, graphs, floats, strings lists, type protos) are counted and skipped
bool parse_attr(const Field& af, MAttr& a) {
  int type = 0;
  Cursor c(af.data, af.len);
  while (!c.done()) {
    Field f = c.next();
    switch (f.num) {
      case 1: a.name = str(f); break;
      case 2: a.f = f32(f); break;
      case 3: a.i = i64(f); break;
      case 4: a.s = str(f); break;
      case 8: rep_i64(f, a.ints); break;
      case 20: type = (int)i64(f); break;
      default: break;
    }
  }
  switch (type) {
    case 0: raise(ONNXB200_ERR_INVALID_MODEL, "undefined attribute type (attribute " + a.name + ")");
    case 1: a.type = ONNXB200_ATTR_FLOAT; return true;
    case 2: a.type = ONNXB200_ATTR_INT; return true;
    case 3: a.type = ONNXB200_ATTR_STRING; return true;
    case 7: a.type = ONNXB200_ATTR_INTS; return true;
    default: return false;
  }
}

// NodeProto (proto/onnx.proto:140-168)
MNode parse_node(const Field& nf, int* skipped_attrs) {
  MNode n;
  Cursor c(nf.data, nf.len);
  while (!c.done()) {
    Field f = c.next();
    switch (f.num) {
      case 1: n.in.push_back(str(f)); break;
      case 2: n.out.push_back(str(f)); break;
      case 3: n.name = str(f); break;
      case 4: n.op = str(f); break;
      case 5: {
        if (f.wire != kLen) raise(ONNXB200_ERR_PROTOBUF, "attribute with wire type " + std::to_string(f.wire));
        MAttr a;
        if (parse_attr(f, a)) n.attrs.push_back(std::move(a));
        else ++*skipped_attrs;
        break;
      }
      case 7: n.domain = str(f); break;
      default: break;
    }
  }
  return n;
}

}  // namespace

struct onnxb200_model {
  int64_t ir_version = 0, opset = 1;
  std::string producer, graph_name, base_dir;
  std::vector<MNode> nodes;
  std::vector<MTensor> inits;       // fp32 initializers
  int skipped_inits = 0, skipped_attrs = 0;
  std::vector<MValue> inputs;       // graph inputs that are not initializers
  std::vector<MValue> outputs;
  // C views handed out by the accessors (pointers into the vectors above)
  std::vector<onnxb200_node> c_nodes;
  std::vector<std::vector<const char*>> c_in, c_out;
  std::vector<std::vector<onnxb200_attr>> c_attrs;
  std::vector<onnxb200_tensor_info> c_inits, c_inputs;
  std::vector<const char*> c_outputs;
};

namespace {

// GraphProto (proto/onnx.proto:108-137)
void parse_graph(const Field& gf, onnxb200_model* m) {
  std::vector<MValue> inputs;
  Cursor c(gf.data, gf.len);
  while (!c.done()) {
    Field f = c.next();
    if (f.wire != kLen) continue;
    switch (f.num) {
      case 1: m->nodes.push_back(parse_node(f, &m->skipped_attrs)); break;
      case 2: m->graph_name = str(f); break;
      case 5: {
        MTensor t = parse_tensor(f);
        if (t.dtype == kFloat) m->inits.push_back(std::move(t));
        else ++m->skipped_inits;
        break;
      }
      case 11: inputs.push_back(parse_value_info(f)); break;
      case 12: m->outputs.push_back(parse_value_info(f)); break;
      default: break;  // value_info, sparse initializers, annotations, doc_string
    }
  }
  // graph inputs may list the initializers too (IR version < 4)
  std::set<std::string> init_names;
  for (auto& t : m->inits) init_names.insert(t.name);
  for (auto& v : inputs)
    if (!init_names.count(v.name)) m->inputs.push_back(std::move(v));
}

// ModelProto (proto/onnx.proto:65-105)
void parse_model(const uint8_t* data, size_t len, onnxb200_model* m) {
  bool have_graph = false;
  bool have_default_domain = false;
  Cursor c(data, len);
  while (!c.done()) {
    Field f = c.next();
    switch (f.num) {
      case 1: m->ir_version = i64(f); break;
      case 2: m->producer = str(f); break;
      case 7:
        if (f.wire != kLen) raise(ONNXB200_ERR_PROTOBUF, "graph with wire type " + std::to_string(f.wire));
        if (have_graph) raise(ONNXB200_ERR_PROTOBUF, "two graphs in one model");
        have_graph = true;
        parse_graph(f, m);
        break;
      case 8: {  // OperatorSetIdProto {domain = 1, version = 2}
        if (f.wire != kLen) raise(ONNXB200_ERR_PROTOBUF, "opset_import with wire type " + std::to_string(f.wire));
        Cursor o(f.data, f.len);
        std::string dom;
        int64_t ver = 1;
        while (!o.done()) {
          Field g = o.next();
          if (g.num == 1) dom = str(g);
          else if (g.num == 2) ver = i64(g);
        }
        if (dom.empty() || (dom == "ai.onnx" && !have_default_domain)) {
          m->opset = ver;
          have_default_domain = have_default_domain || dom.empty();
        }
        break;
      }
      default: break;
    }
  }
  if (!have_graph) raise(ONNXB200_ERR_INVALID_MODEL, "Model is missing graph");
}

void load_external(onnxb200_model* m) {
  for (auto& t : m->inits) {
    if (!t.external) continue;
    if (m->base_dir.empty())
      raise(ONNXB200_ERR_UNSUPPORTED, "tensor " + t.name + " has external data; load the model from its file");
    if (t.location.find("..") != std::string::npos || (!t.location.empty() && t.location[0] == '/'))
      raise(ONNXB200_ERR_INVALID_MODEL, "external data location outside the model's directory: " + t.location);
    const std::string path = m->base_dir + "/" + t.location;
    std::ifstream in(path, std::ios::binary);
    if (!in) raise(ONNXB200_ERR_IO, "cannot open external data file " + path);
    const int64_t n = numel(t.dims);
    t.data.resize((size_t)n);
    in.seekg(t.offset);
    in.read(reinterpret_cast<char*>(t.data.data()), n * 4);
    if (!in || in.gcount() != n * 4) raise(ONNXB200_ERR_IO, "external data file " + path + " is too short");
    t.have_data = true;
    t.external = false;
  }
}

void build_views(onnxb200_model* m) {
  const size_t nn = m->nodes.size();
  m->c_in.resize(nn);
  m->c_out.resize(nn);
  m->c_attrs.resize(nn);
  m->c_nodes.resize(nn);
  for (size_t k = 0; k < nn; ++k) {
    MNode& n = m->nodes[k];
    for (auto& s : n.in) m->c_in[k].push_back(s.c_str());
    for (auto& s : n.out) m->c_out[k].push_back(s.c_str());
    for (auto& a : n.attrs) {
      onnxb200_attr ca{};
      ca.name = a.name.c_str();
      ca.type = a.type;
      ca.i = a.i;
      ca.f = a.f;
      ca.ints = a.ints.data();
      ca.n_ints = (int)a.ints.size();
      ca.s = a.s.c_str();
      m->c_attrs[k].push_back(ca);
    }
    onnxb200_node& c = m->c_nodes[k];
    c.op_type = n.op.c_str();
    c.inputs = m->c_in[k].data();
    c.n_inputs = (int)n.in.size();
    c.outputs = m->c_out[k].data();
    c.n_outputs = (int)n.out.size();
    c.attrs = m->c_attrs[k].data();
    c.n_attrs = (int)n.attrs.size();
  }
  for (auto& t : m->inits) {
    onnxb200_tensor_info ti{};
    ti.name = t.name.c_str();
    ti.data = t.data.data();
    ti.shape = t.dims.data();
    ti.rank = (int)t.dims.size();
    m->c_inits.push_back(ti);
  }
  for (auto& v : m->inputs) {
    onnxb200_tensor_info ti{};
    ti.name = v.name.c_str();
    ti.shape = v.dims.data();
    ti.rank = (int)v.dims.size();
    m->c_inputs.push_back(ti);
  }
  for (auto& v : m->outputs) m->c_outputs.push_back(v.name.c_str());
}

void set_err(char* err, size_t err_len, const std::string& msg) {
  if (!err || !err_len) return;
  std::snprintf(err, err_len, "%s", msg.c_str());
}

int parse_into(const uint8_t* data, size_t len, const std::string& base_dir, onnxb200_model** out, char* err,
               size_t err_len) {
  onnxb200_model* m = new (std::nothrow) onnxb200_model;
  if (!m) return ONNXB200_ERR_RESOURCE_EXHAUSTED;
  m->base_dir = base_dir;
  try {
    parse_model(data, len, m);
    load_external(m);
    build_views(m);
  } catch (const ParseError& e) {
    set_err(err, err_len, e.msg);
    delete m;
    return e.code;
  } catch (const std::bad_alloc&) {
    set_err(err, err_len, "out of host memory while reading the model");
    delete m;
    return ONNXB200_ERR_RESOURCE_EXHAUSTED;
  }
  *out = m;
  return ONNXB200_OK;
}

}  // namespace

extern "C" ONNXB200_API int onnxb200_model_parse(const void* data, size_t len, const char* base_dir,
                                                 onnxb200_model** out, char* err, size_t err_len) {
  if (!out || (!data && len)) return ONNXB200_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  return parse_into(static_cast<const uint8_t*>(data), len, base_dir ? base_dir : "", out, err, err_len);
}

extern "C" ONNXB200_API int onnxb200_model_load(const char* path, onnxb200_model** out, char* err,
                                                size_t err_len) {
  if (!path || !out) return ONNXB200_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  if (!in) {
    set_err(err, err_len, std::string("Failed to open file: ") + path);
    return ONNXB200_ERR_IO;
  }
  const std::streamoff n = in.tellg();
  std::vector<uint8_t> buf;
  try {
    buf.resize((size_t)n);
  } catch (const std::bad_alloc&) {
    set_err(err, err_len, "out of host memory while reading the model");
    return ONNXB200_ERR_RESOURCE_EXHAUSTED;
  }
  in.seekg(0);
  if (n && !in.read(reinterpret_cast<char*>(buf.data()), n)) {
    set_err(err, err_len, std::string("Failed to read file: ") + path);
    return ONNXB200_ERR_IO;
  }
  std::string dir(path);
  const size_t slash = dir.find_last_of('/');
  dir = slash == std::string::npos ? std::string(".") : dir.substr(0, slash == 0 ? 1 : slash);
  return parse_into(buf.data(), buf.size(), dir, out, err, err_len);
}

extern "C" ONNXB200_API int onnxb200_model_get_info(const onnxb200_model* m, onnxb200_model_info* info) {
  if (!m || !info) return ONNXB200_ERR_INVALID_ARGUMENT;
  info->ir_version = m->ir_version;
  info->opset = m->opset;
  info->n_nodes = (int)m->nodes.size();
  info->n_initializers = (int)m->inits.size();
  info->n_skipped_initializers = m->skipped_inits;
  info->n_skipped_attributes = m->skipped_attrs;
  info->n_inputs = (int)m->inputs.size();
  info->n_outputs = (int)m->outputs.size();
  info->producer_name = m->producer.c_str();
  info->graph_name = m->graph_name.c_str();
  return ONNXB200_OK;
}

extern "C" ONNXB200_API int onnxb200_model_get_nodes(const onnxb200_model* m, const onnxb200_node** nodes,
                                                     int* n) {
  if (!m || !nodes || !n) return ONNXB200_ERR_INVALID_ARGUMENT;
  *nodes = m->c_nodes.data();
  *n = (int)m->c_nodes.size();
  return ONNXB200_OK;
}

extern "C" ONNXB200_API int onnxb200_model_get_initializers(const onnxb200_model* m,
                                                            const onnxb200_tensor_info** t, int* n) {
  if (!m || !t || !n) return ONNXB200_ERR_INVALID_ARGUMENT;
  *t = m->c_inits.data();
  *n = (int)m->c_inits.size();
  return ONNXB200_OK;
}

extern "C" ONNXB200_API int onnxb200_model_get_inputs(const onnxb200_model* m, const onnxb200_tensor_info** t,
                                                      int* n) {
  if (!m || !t || !n) return ONNXB200_ERR_INVALID_ARGUMENT;
  *t = m->c_inputs.data();
  *n = (int)m->c_inputs.size();
  return ONNXB200_OK;
}

extern "C" ONNXB200_API int onnxb200_model_get_outputs(const onnxb200_model* m, const char* const** names,
                                                       int* n) {
  if (!m || !names || !n) return ONNXB200_ERR_INVALID_ARGUMENT;
  *names = m->c_outputs.data();
  *n = (int)m->c_outputs.size();
  return ONNXB200_OK;
}

extern "C" ONNXB200_API int onnxb200_model_destroy(onnxb200_model* m) {
  delete m;
  return ONNXB200_OK;
}

extern "C" ONNXB200_API int onnxb200_graph_build_from_model(onnxb200_handle* h, const onnxb200_model* m,
                                                            const onnxb200_tensor_info* input_shapes,
                                                            int n_input_shapes, onnxb200_graph** out) {
  if (!h || !m || !out || n_input_shapes < 0 || (n_input_shapes && !input_shapes))
    return ONNXB200_ERR_INVALID_ARGUMENT;
  std::vector<onnxb200_tensor_info> ins(m->c_inputs);
  for (int k = 0; k < n_input_shapes; ++k) {
    const onnxb200_tensor_info& o = input_shapes[k];
    bool found = false;
    for (auto& t : ins)
      if (o.name && std::strcmp(o.name, t.name) == 0) {
        t.shape = o.shape;
        t.rank = o.rank;
        found = true;
      }
    if (!found)
      return ob2::set_error(h, ONNXB200_ERR_VALIDATION,
                            std::string("input shape given for ") + (o.name ? o.name : "(null)") +
                                ", which is not a graph input");
  }
  for (auto& t : ins)
    for (int d = 0; d < t.rank; ++d)
      if (t.shape[d] <= 0)
        return ob2::set_error(h, ONNXB200_ERR_VALIDATION,
                              std::string("graph input ") + t.name +
                                  " has a symbolic or empty dimension: pass its shape");
  return onnxb200_graph_build(h, m->c_nodes.data(), (int)m->c_nodes.size(), m->c_inits.data(),
                              (int)m->c_inits.size(), ins.data(), (int)ins.size(), m->c_outputs.data(),
                              (int)m->c_outputs.size(), out);
}
