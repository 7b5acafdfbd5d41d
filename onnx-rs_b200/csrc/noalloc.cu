// Convolution entry point that allocates no device memory.
//
// Who needs it: callers that must not call cudaMalloc while they run -- for
// example a host framework that hands this library pre-sized input and output
// buffers from its own arena and forbids allocation inside an operator, or a
// latency-critical serving loop that cannot afford an allocation (or the
// implicit device synchronisation cudaFree brings).  The regular entry point
// onnxb200_conv2d needs scratch memory for the packed weights and takes it
// from the handle's workspace, which it grows with cudaMalloc on demand, and a
// handle itself is created with cudaMalloc.
//
// This variant takes a stream instead of a handle and puts its scratch (the
// tf32 hi/lo packed weights, the folded BatchNormalization / bias vectors and a
// status word) in one fixed, file-scope device array.  Every GPU that loads
// the library holds that array until the process exits.
#include <cuda_runtime.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "internal.h"

namespace {

constexpr size_t kScratchBytes = ONNXB200_NOALLOC_SCRATCH_BYTES;
constexpr size_t kStatusBytes = 256;  // status word at the front, weights after it

// Shared by every call on a device; holds the previous call's contents.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
struct DeviceState {
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch
  int num_sms = 0;
  // Recorded on the caller's stream after each call's kernels: the next call
  // waits for it (bounded) before it rewrites the array, so a call that gave up
  // waiting (ONNXB200_ERR_TIMEOUT) never has its packed weights overwritten
  // while its kernels still read them.
  cudaEvent_t done = nullptr;
  // A non-blocking stream of the library's own for reading the status word, so
  // that the read waits neither for the caller's later work nor for other
  // threads' work on the legacy default stream.
  cudaStream_t status_stream = nullptr;
};
DeviceState g_dev[kMaxDevices];

// Host code cannot use g_noalloc_scratch as a pointer (it names the host-side
// shadow of the symbol), so the device address is looked up once per device,
// with that device current.  The event and stream are created then too (neither
// allocates device memory).
int setup_device(int dev, DeviceState** out) {
  if (dev < 0 || dev >= kMaxDevices) return ONNXB200_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  DeviceState& st = g_dev[dev];
  if (!st.scratch) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return ONNXB200_ERR_EXECUTION;
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return ONNXB200_ERR_EXECUTION;
    if (!st.done && cudaEventCreateWithFlags(&st.done, cudaEventDisableTiming) != cudaSuccess)
      return ONNXB200_ERR_EXECUTION;
    if (!st.status_stream &&
        cudaStreamCreateWithFlags(&st.status_stream, cudaStreamNonBlocking) != cudaSuccess)
      return ONNXB200_ERR_EXECUTION;
    st.num_sms = sms;
    st.scratch = static_cast<unsigned char*>(p);
  }
  *out = &st;
  return ONNXB200_OK;
}

// Polls `ev` until it has completed or `timeout_ms` passed.
int wait_event_bounded(cudaEvent_t ev, int timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return ONNXB200_OK;
    if (q != cudaErrorNotReady) return ONNXB200_ERR_EXECUTION;
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
      return ONNXB200_ERR_TIMEOUT;
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

}  // namespace

extern "C" int onnxb200_conv2d_nhwc_noalloc(void* cuda_stream, const onnxb200_conv_desc* d,
                                            const float* x, const float* w, const float* bias,
                                            const float* bn_scale, const float* bn_bias,
                                            const float* bn_mean, const float* bn_var,
                                            const float* residual, float* y) {
  if (!d) return ONNXB200_ERR_INVALID_ARGUMENT;
  if (d->layout != ONNXB200_LAYOUT_NHWC) return ONNXB200_ERR_VALIDATION;  // NCHW would need repack scratch
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ONNXB200_ERR_EXECUTION;
  // The call blocks until y is written, which a capturing stream cannot do.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(static_cast<cudaStream_t>(cuda_stream), &cap) != cudaSuccess)
    return ONNXB200_ERR_EXECUTION;
  if (cap != cudaStreamCaptureStatusNone) return ONNXB200_ERR_UNSUPPORTED;
  DeviceState* ds = nullptr;
  int rc = setup_device(dev, &ds);
  if (rc) return rc;
  unsigned char* scratch = ds->scratch;
  constexpr int kTimeoutMs = 60000;

  // A handle-shaped view over the caller's stream and the fixed scratch; no
  // device memory is allocated for it.
  onnxb200_handle view;
  view.device = dev;
  view.num_sms = ds->num_sms;
  view.stream = static_cast<cudaStream_t>(cuda_stream);
  view.own_stream = nullptr;
  view.d_status = reinterpret_cast<int*>(scratch);
  view.opts.precision = ONNXB200_PREC_3XTF32;
  view.opts.wait_timeout_ms = kTimeoutMs;

  onnxb200_conv_desc r;
  int64_t oh = 0, ow = 0;
  rc = ob2::resolve_conv_desc(&view, d, &r, &oh, &ow);
  if (rc) return rc;
  if (r.n == 0) return ONNXB200_OK;
  if (!x || !w || !y) return ONNXB200_ERR_INVALID_ARGUMENT;

  // Size check before touching the device: everything must fit the array.
  onnxb200_conv_plan plan;
  size_t need = 0;
  rc = ob2::conv_plan_init(&view, d, (int)r.c, w, bias, bn_scale, bn_bias, bn_mean, bn_var, &plan,
                           nullptr, 0, &need);
  if (rc) return rc;
  if (need > kScratchBytes - kStatusBytes) return ONNXB200_ERR_RESOURCE_EXHAUSTED;

  // The previous call on this device (possibly one that timed out) must be
  // done with the array before it is rewritten.
  rc = wait_event_bounded(ds->done, kTimeoutMs);
  if (rc) return rc;

  // The status word must start at zero; the packed weights and epilogue
  // vectors are fully rewritten below, so the rest needs no clearing.
  if (cudaMemsetAsync(view.d_status, 0, sizeof(int), view.stream) != cudaSuccess)
    return ONNXB200_ERR_EXECUTION;
  size_t used = 0;
  rc = ob2::conv_plan_init(&view, d, (int)r.c, w, bias, bn_scale, bn_bias, bn_mean, bn_var, &plan,
                           scratch + kStatusBytes, kScratchBytes - kStatusBytes, &used);
  if (rc == ONNXB200_OK) rc = ob2::conv_plan_exec_nhwc(&view, &plan, x, residual, y);
  // recorded even after a failed launch, so the next call's wait ends
  if (cudaEventRecord(ds->done, view.stream) != cudaSuccess) return ONNXB200_ERR_EXECUTION;
  if (rc) return rc;

  // Blocking: return once y is written, so that sequential calls never share
  // the array while one of them is still running.  The wait is bounded; after
  // a timeout the next call first waits for this one's kernels.
  rc = wait_event_bounded(ds->done, kTimeoutMs);
  if (rc) return rc;
  int status = 0;
  if (cudaMemcpyAsync(&status, view.d_status, sizeof(int), cudaMemcpyDeviceToHost, ds->status_stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(ds->status_stream) != cudaSuccess)
    return ONNXB200_ERR_EXECUTION;
  return status;
}
