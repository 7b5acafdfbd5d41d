// Batch-sharded replicas of one graph on several GPUs of this process.
//
// Inference on a batch is embarrassingly parallel over the batch: each GPU
// holds its own copy of the packed weights and runs its contiguous slice of the
// images; there is no collective.  The reference has no multi-device path (its
// concurrency is rayon over the nodes of one graph on host cores,
// ExecutionEngine::run_concurrent, src/execution/engine.rs:743-809); this is the
// device-side counterpart for a batch.
//
//   build:  one host thread per device creates that device's handle and builds
//           the graph with the slice's batch (the slices differ by at most one
//           image), all devices in parallel.
//   run:    one host thread per device copies its slice of each host input in,
//           replays its captured graph and copies its slice of each output into
//           the disjoint rows of the caller's host output buffers; the threads
//           start together from a host barrier, and each device's time from
//           that release to its last completion event is kept (CUDA events).
#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "internal.h"

namespace {

// Start line for the worker threads of one run: every thread waits until all
// have arrived, so that the devices start together.
class StartBarrier {
 public:
  explicit StartBarrier(int n) : n_(n) {}
  void arrive_and_wait() {
    std::unique_lock<std::mutex> lock(m_);
    if (++count_ == n_) {
      cv_.notify_all();
      return;
    }
    cv_.wait(lock, [&] { return count_ >= n_; });
  }

 private:
  std::mutex m_;
  std::condition_variable cv_;
  int n_, count_ = 0;
};

struct Replica {
  int device = 0;
  int64_t lo = 0, hi = 0;  // batch rows [lo, hi)
  onnxb200_handle* h = nullptr;
  onnxb200_graph* g = nullptr;
  cudaEvent_t ev_start = nullptr, ev_end = nullptr;
  float last_ms = 0.f;
};

}  // namespace

struct onnxb200_multi {
  std::vector<Replica> reps;
  int64_t batch = 0;
  std::vector<int64_t> in_row, out_row;  // elements per batch row of each input / output
  std::vector<std::vector<int64_t>> out_shapes;  // full-batch output shapes
  std::string last_error;
};

namespace {

void set_err(char* err, size_t len, const std::string& m) {
  if (err && len) {
    std::strncpy(err, m.c_str(), len - 1);
    err[len - 1] = 0;
  }
}

void destroy_multi(onnxb200_multi* m) {
  if (!m) return;
  for (Replica& r : m->reps) {
    if (r.g) onnxb200_graph_destroy(r.g);
    if (r.ev_start || r.ev_end) cudaSetDevice(r.device);
    if (r.ev_start) cudaEventDestroy(r.ev_start);
    if (r.ev_end) cudaEventDestroy(r.ev_end);
    if (r.h) onnxb200_destroy(r.h);
  }
  delete m;
}

}  // namespace

extern "C" int onnxb200_multi_build(const int* devices, int n_devices, const onnxb200_options* opts,
                                    const onnxb200_node* nodes, int n_nodes,
                                    const onnxb200_tensor_info* initializers, int n_init,
                                    const onnxb200_tensor_info* inputs, int n_inputs, const char* const* outputs,
                                    int n_outputs, onnxb200_multi** out, char* err, size_t err_len) {
  set_err(err, err_len, "");
  if (!devices || n_devices <= 0 || !out || n_inputs <= 0 || !inputs || n_outputs <= 0 || !outputs) {
    set_err(err, err_len, "onnxb200_multi_build: null or empty argument");
    return ONNXB200_ERR_INVALID_ARGUMENT;
  }
  *out = nullptr;
  // every graph input is split along its first dimension: one batch for all
  int64_t batch = -1;
  for (int i = 0; i < n_inputs; ++i) {
    if (!inputs[i].shape || inputs[i].rank < 1) {
      set_err(err, err_len, "onnxb200_multi_build: graph inputs need a batch dimension");
      return ONNXB200_ERR_VALIDATION;
    }
    if (batch < 0) batch = inputs[i].shape[0];
    if (inputs[i].shape[0] != batch) {
      set_err(err, err_len, "onnxb200_multi_build: graph inputs disagree on the batch size");
      return ONNXB200_ERR_VALIDATION;
    }
  }
  if (batch < n_devices) {
    set_err(err, err_len, "onnxb200_multi_build: fewer images than devices");
    return ONNXB200_ERR_VALIDATION;
  }
  for (int i = 0; i < n_devices; ++i)
    for (int j = 0; j < i; ++j)
      if (devices[i] == devices[j]) {
        set_err(err, err_len, "onnxb200_multi_build: a device is listed twice");
        return ONNXB200_ERR_VALIDATION;
      }
  onnxb200_multi* m = new (std::nothrow) onnxb200_multi();
  if (!m) return ONNXB200_ERR_RESOURCE_EXHAUSTED;
  m->batch = batch;
  m->reps.resize(n_devices);
  for (int d = 0; d < n_devices; ++d) {
    Replica& r = m->reps[d];
    r.device = devices[d];
    // contiguous slices, the first batch % n devices one image larger
    const int64_t base = batch / n_devices, extra = batch % n_devices;
    r.lo = d * base + std::min<int64_t>(d, extra);
    r.hi = r.lo + base + (d < extra ? 1 : 0);
  }
  for (int i = 0; i < n_inputs; ++i) {
    int64_t row = 1;
    for (int k = 1; k < inputs[i].rank; ++k) row *= inputs[i].shape[k];
    m->in_row.push_back(row);
  }
  // per device: handle + graph with the slice's batch, built in parallel
  std::vector<int> rc(n_devices, ONNXB200_OK);
  std::vector<std::string> msg(n_devices);
  std::vector<std::thread> th;
  for (int d = 0; d < n_devices; ++d)
    th.emplace_back([&, d] {
      Replica& r = m->reps[d];
      rc[d] = onnxb200_create(r.device, opts, &r.h);
      if (rc[d]) {
        msg[d] = "device " + std::to_string(r.device) + ": handle creation failed";
        return;
      }
      std::vector<std::vector<int64_t>> shp(n_inputs);
      std::vector<onnxb200_tensor_info> ins(inputs, inputs + n_inputs);
      for (int i = 0; i < n_inputs; ++i) {
        shp[i].assign(inputs[i].shape, inputs[i].shape + inputs[i].rank);
        shp[i][0] = r.hi - r.lo;
        ins[i].shape = shp[i].data();
      }
      rc[d] = onnxb200_graph_build(r.h, nodes, n_nodes, initializers, n_init, ins.data(), n_inputs, outputs,
                                   n_outputs, &r.g);
      if (rc[d]) {
        msg[d] = "device " + std::to_string(r.device) + ": " + onnxb200_last_error(r.h);
        return;
      }
      if (cudaSetDevice(r.device) != cudaSuccess || cudaEventCreate(&r.ev_start) != cudaSuccess ||
          cudaEventCreate(&r.ev_end) != cudaSuccess) {
        rc[d] = ONNXB200_ERR_EXECUTION;
        msg[d] = "device " + std::to_string(r.device) + ": event creation failed";
      }
    });
  for (auto& t : th) t.join();
  for (int d = 0; d < n_devices; ++d)
    if (rc[d]) {
      set_err(err, err_len, msg[d]);
      destroy_multi(m);
      return rc[d];
    }
  // outputs: every one must carry the batch in its first dimension
  for (int o = 0; o < n_outputs; ++o) {
    std::vector<int64_t> shape;
    for (int d = 0; d < n_devices; ++d) {
      int64_t s[16];
      int rank = 0;
      if (onnxb200_graph_output_shape(m->reps[d].g, o, s, &rank) != ONNXB200_OK || rank < 1 || rank > 16 ||
          s[0] != m->reps[d].hi - m->reps[d].lo) {
        set_err(err, err_len, std::string("onnxb200_multi_build: output ") + outputs[o] +
                                  " does not have the batch as its first dimension");
        destroy_multi(m);
        return ONNXB200_ERR_UNSUPPORTED;
      }
      if (d == 0) shape.assign(s, s + rank);
    }
    shape[0] = batch;
    int64_t row = 1;
    for (size_t k = 1; k < shape.size(); ++k) row *= shape[k];
    m->out_row.push_back(row);
    m->out_shapes.push_back(shape);
  }
  *out = m;
  return ONNXB200_OK;
}

extern "C" int onnxb200_multi_run_host(onnxb200_multi* m, int n_batches, const float* const* inputs,
                                       float* const* outputs) {
  if (!m || n_batches < 0 || (n_batches > 0 && (!inputs || !outputs))) return ONNXB200_ERR_INVALID_ARGUMENT;
  if (n_batches == 0) return ONNXB200_OK;
  const size_t ni = m->in_row.size(), no = m->out_row.size();
  const int nd = (int)m->reps.size();
  std::vector<int> rc(nd, ONNXB200_OK);
  StartBarrier start(nd);
  std::vector<std::thread> th;
  for (int d = 0; d < nd; ++d)
    th.emplace_back([&, d] {
      Replica& r = m->reps[d];
      // this device's slice of every batch's inputs and outputs
      std::vector<const float*> in(n_batches * ni);
      std::vector<float*> outp(n_batches * no);
      for (int b = 0; b < n_batches; ++b) {
        for (size_t i = 0; i < ni; ++i) in[b * ni + i] = inputs[b * ni + i] + r.lo * m->in_row[i];
        for (size_t o = 0; o < no; ++o) outp[b * no + o] = outputs[b * no + o] + r.lo * m->out_row[o];
      }
      cudaSetDevice(r.device);
      // nothing of an earlier call may still be running when the clock starts
      int e = onnxb200_synchronize(r.h);
      start.arrive_and_wait();
      if (e) {
        rc[d] = e;
        return;
      }
      cudaStream_t st = static_cast<cudaStream_t>(onnxb200_get_stream(r.h));
      cudaEventRecord(r.ev_start, st);
      e = onnxb200_graph_run_host_pipelined(r.h, r.g, n_batches, in.data(), outp.data());
      cudaEventRecord(r.ev_end, st);
      if (!e && cudaEventSynchronize(r.ev_end) != cudaSuccess) e = ONNXB200_ERR_EXECUTION;
      if (!e) cudaEventElapsedTime(&r.last_ms, r.ev_start, r.ev_end);
      rc[d] = e;
    });
  for (auto& t : th) t.join();
  for (int d = 0; d < nd; ++d)
    if (rc[d]) {
      m->last_error = "device " + std::to_string(m->reps[d].device) + ": " + onnxb200_last_error(m->reps[d].h);
      return rc[d];
    }
  m->last_error.clear();
  return ONNXB200_OK;
}

extern "C" int onnxb200_multi_get_info(const onnxb200_multi* m, int* n_devices, int64_t* batch,
                                       int64_t* slice_begin, float* last_run_ms) {
  if (!m) return ONNXB200_ERR_INVALID_ARGUMENT;
  if (n_devices) *n_devices = (int)m->reps.size();
  if (batch) *batch = m->batch;
  for (size_t d = 0; d < m->reps.size(); ++d) {
    if (slice_begin) slice_begin[d] = m->reps[d].lo;
    if (last_run_ms) last_run_ms[d] = m->reps[d].last_ms;
  }
  return ONNXB200_OK;
}

extern "C" int onnxb200_multi_output_shape(const onnxb200_multi* m, int index, int64_t* shape, int* rank) {
  if (!m || !rank || index < 0 || index >= (int)m->out_shapes.size()) return ONNXB200_ERR_INVALID_ARGUMENT;
  const auto& s = m->out_shapes[index];
  *rank = (int)s.size();
  if (shape) std::copy(s.begin(), s.end(), shape);
  return ONNXB200_OK;
}

extern "C" const char* onnxb200_multi_last_error(const onnxb200_multi* m) {
  return m ? m->last_error.c_str() : "null multi-device graph";
}

extern "C" int onnxb200_multi_destroy(onnxb200_multi* m) {
  if (!m) return ONNXB200_ERR_INVALID_ARGUMENT;
  destroy_multi(m);
  return ONNXB200_OK;
}
