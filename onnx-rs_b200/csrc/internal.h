// Host-side internals shared by api.cpp and graph.cpp.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/onnxb200.h"
#include "kernels.h"

struct onnxb200_handle {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  onnxb200_options opts{};
  void* ws = nullptr;        // workspace (grows on demand, stream-ordered reuse)
  size_t ws_bytes = 0;
  int* d_status = nullptr;   // device status word written by kernels
  float* d_ones = nullptr;   // scratch constants
  std::string last_error;
  int64_t launches = 0;
  // ONNXB200_DEBUG_SYNC=1: graph runs synchronize after every step and report
  // the first step whose kernels failed (eager runs only).
  bool debug_sync = false;
};

struct onnxb200_conv_plan {
  onnxb200_conv_desc d{};    // pads resolved, precision resolved
  int64_t oh = 0, ow = 0;
  int prec = 0;
  bool use_tc = false;       // tcgen05 implicit GEMM (else CUDA-core direct conv)
  int cs_in = 0;             // channel stride of the NHWC input the plan expects
  int K = 0, num_kb = 0, kpad = 0, bn = 128;
  void* w_hi = nullptr;      // packed weights (tc path)
  void* w_lo = nullptr;
  float* w_oihw = nullptr;   // original weights (CUDA-core path)
  float* scale = nullptr;    // epilogue per-channel multiplier (BN) or null
  float* shift = nullptr;    // epilogue per-channel addend (bias / BN) or null
  CUtensorMap tm_hi{}, tm_lo{};
  int64_t weight_bytes = 0;
  // Pixel pairs (4-channel input, horizontal stride 2, even width): the NHWC
  // input is read as [N][H][W/2][8] and the convolution runs with stride 1 over
  // ceil((KW + pw%2)/2) pair taps -- the same memory, half the TMA box rows.
  bool pairs = false;
  // BF16 precision in a graph: the input activations (x, x2) are stored as bf16
  // (64-element k-blocks), and / or the output and residual are.
  bool a_bf16 = false;
  bool out_bf16 = false;
  // Two sources (conv_dual_plan_init): a 1x1 stride-1 convolution of x (this
  // descriptor) plus a 1x1 convolution of x2 (d2, stride d2.stride_h) at the
  // same output pixels, weights packed side by side along K with each branch's
  // folded BatchNormalization scale, shift = both branches' shifts.
  bool dual = false;
  onnxb200_conv_desc d2{};
  int cs2 = 0;
  int kb_split = 0;
  // K split (igemm_launch_split) when the problem has too few output tiles to
  // fill the GPU: `ksplit` slices, partial sums in a buffer of split_bytes --
  // the plan's own (split_ws, op-level plans) or one the caller passes (graphs);
  // with neither the plan runs unsplit.
  int ksplit = 1;
  int split_mt = 0;          // first split M-tile (0 = all; > 0: only the last wave's)
  size_t split_bytes = 0;
  float* split_ws = nullptr;
};

namespace ob2 {

int set_error(onnxb200_handle* h, int code, const std::string& msg);
int cuda_check(onnxb200_handle* h, cudaError_t e, const char* what);
int ensure_workspace(onnxb200_handle* h, size_t bytes);

// Encodes a 2-D TMA map over a [rows][kpad] K-major weight matrix.
int encode_weight_map(onnxb200_handle* h, CUtensorMap* map, const void* base, int rows, int kpad,
                      int prec, int bn, int bk = 32);

// Resolves auto_pad / defaults and validates a conv descriptor.
int resolve_conv_desc(onnxb200_handle* h, const onnxb200_conv_desc* in, onnxb200_conv_desc* out,
                      int64_t* oh, int64_t* ow);

// Builds a conv plan whose weights live in memory owned by the plan (cudaMalloc)
// or, when `scratch` is non-null, inside the given scratch region (no allocation).
// With scratch == nullptr and scratch_used != nullptr it only reports the bytes
// the plan needs.
int conv_plan_init(onnxb200_handle* h, const onnxb200_conv_desc* d, int cs_in, const float* w,
                   const float* bias, const float* bn_scale, const float* bn_bias,
                   const float* bn_mean, const float* bn_var, onnxb200_conv_plan* p,
                   void* scratch, size_t scratch_bytes, size_t* scratch_used, bool a_bf16 = false,
                   bool out_bf16 = false);
void conv_plan_free(onnxb200_conv_plan* p);

// BatchNormalization of one branch of a two-source convolution (all device
// pointers; conv_bias may be null).
struct ConvBranchBN {
  const float* scale = nullptr;
  const float* bias = nullptr;
  const float* mean = nullptr;
  const float* var = nullptr;
  const float* conv_bias = nullptr;
  float eps = 1e-5f;
};
// Whether y = BN1(conv1(x1)) + BN2(conv2(x2)) can run as one two-source
// problem: both 1x1 pad-0 convolutions with channel counts that are multiples
// of 32 and no channel padding, conv1 of stride 1, the same output shape and a
// tensor-core precision.
bool dual_conv_supported(const onnxb200_conv_desc& d1, int cs1, const onnxb200_conv_desc& d2, int cs2);
int conv_dual_plan_init(onnxb200_handle* h, const onnxb200_conv_desc* d1, int cs1, const float* w1,
                        const ConvBranchBN& bn1, const onnxb200_conv_desc* d2, int cs2, const float* w2,
                        const ConvBranchBN& bn2, onnxb200_conv_plan* p, void* scratch, size_t scratch_bytes,
                        size_t* scratch_used, bool a_bf16 = false, bool out_bf16 = false);
int conv_dual_exec_nhwc(onnxb200_handle* h, const onnxb200_conv_plan* p, const float* x1, const float* x2,
                        float* y, float* split_ws = nullptr);

// Runs a plan on NHWC buffers (x channel stride p->cs_in, y / residual stride C_out).
// split_ws (>= p->split_bytes, or null for the plan's own) holds K-split partial sums.
int conv_plan_exec_nhwc(onnxb200_handle* h, const onnxb200_conv_plan* p, const float* x,
                        const float* residual, float* y, float* split_ws = nullptr);

// Plain GEMM on the tcgen05 core:  y[b] = A_b * B_b^T(packed) with epilogue.
struct GemmCall {
  const float* a = nullptr;  // row-major [M][K] per batch, lda == K
  int M = 0, N = 0, K = 0;
  int a_rows = 0;            // rows of the whole A array (all batches); 0 = M
  int batches = 1;
  const long long* a_off = nullptr;  // device array or null
  const int* b_row = nullptr;        // device array or null
  long long y_bstride = 0;
  float* y = nullptr;
  int ldy = 0;
  const float* scale = nullptr;
  const float* shift = nullptr;
  const float* res = nullptr;
  int ldr = 0;
  int relu = 0;
  // K-split buffer (may be null): used when a split is modelled faster and fits
  float* split_ws = nullptr;
  size_t split_bytes = 0;
};
int gemm_tc_run(onnxb200_handle* h, const GemmCall& c, const void* b_hi, const void* b_lo,
                int b_rows, int kpad, int prec);
// Bytes of K-split buffer a single-batch tensor-core GEMM of this shape would
// use in gemm_tc_run (0 = it would not split).
size_t gemm_split_bytes(const onnxb200_handle* h, int M, int N, int kpad, int prec, bool residual);

inline int resolve_prec(const onnxb200_handle* h, int prec) {
  return prec < 0 ? h->opts.precision : prec;
}

}  // namespace ob2
