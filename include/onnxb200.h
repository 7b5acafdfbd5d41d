/*
 * onnxb200 -- C ABI of the B200 (sm_100a) Conv / MatMul / Gemm / pooling path.
 *
 * This is the drop-in boundary for the onnx-rs operator interface
 * (src/ops/registry.rs:14-27, trait Operator { compute, output_shapes,
 * validate }).  Each entry point below names the reference function or trait
 * method it replaces.  Plain pointers and sizes only: tensors are caller-owned
 * DEVICE buffers of fp32 unless stated otherwise; nothing in these signatures
 * is a torch or Rust type.
 *
 * Conventions
 *  - Every function returns an onnxb200 status code (0 = OK).  Codes map 1:1 to
 *    the reference's crate::error::Error variants (src/error.rs:19-66).  No C++
 *    exception and no abort crosses this boundary.  After a failure,
 *    onnxb200_last_error(handle) gives a message.
 *  - A handle owns one CUDA stream, a stream-ordered workspace and a device
 *    status word.  All compute calls are asynchronous on the handle's stream;
 *    onnxb200_synchronize waits (bounded by the handle's wait_timeout_ms) and
 *    reports device-side failures (e.g. ONNXB200_ERR_TIMEOUT from a kernel
 *    whose internal wait gave up).  Use one handle per host thread per GPU, as
 *    the reference's operators are called from rayon workers
 *    (src/execution/engine.rs:800-809) without sharing mutable state.
 *  - Activations are NCHW (the reference layout, src/ops/tensor.rs:206-218) or
 *    NHWC, chosen per call by a layout field; weights are OIHW as in ONNX.
 */
#ifndef ONNXB200_H
#define ONNXB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ONNXB200_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- status codes */
/* (values are also defined, identically, in onnx-rs_b200/csrc/status.h) */
#ifndef ONNXB200_OK
#define ONNXB200_OK 0
#define ONNXB200_ERR_VALIDATION 1         /* Error::ValidationError */
#define ONNXB200_ERR_EXECUTION 2          /* Error::ExecutionError (CUDA error) */
#define ONNXB200_ERR_UNSUPPORTED 3        /* Error::UnsupportedFeature */
#define ONNXB200_ERR_TIMEOUT 4            /* Error::OperationTimeout */
#define ONNXB200_ERR_RESOURCE_EXHAUSTED 5 /* Error::ResourceExhausted */
#define ONNXB200_ERR_INVALID_GRAPH 6      /* Error::InvalidGraph */
#define ONNXB200_ERR_INVALID_OPERATOR 7   /* Error::InvalidOperator */
#define ONNXB200_ERR_CANCELLED 8          /* Error::ExecutionCancelled */
#define ONNXB200_ERR_INVALID_ARGUMENT 9   /* null handle / pointer */
#define ONNXB200_ERR_IO 10                /* Error::IoError / Error::ModelLoadError */
#define ONNXB200_ERR_PROTOBUF 11          /* Error::ProtobufError (malformed model bytes) */
#define ONNXB200_ERR_INVALID_MODEL 12     /* Error::InvalidModel / Error::MissingField */
#endif

/* ---------------------------------------------------------------- enums */
/* Arithmetic of the contractions (Conv, MatMul, Gemm). */
#define ONNXB200_PREC_DEFAULT (-1)  /* use the handle's default */
#define ONNXB200_PREC_3XTF32 0      /* tcgen05 3xTF32 split: fp32-accurate (default) */
#define ONNXB200_PREC_TF32 1        /* tcgen05 1xTF32 (fast mode) */
#define ONNXB200_PREC_BF16 2        /* tcgen05 bf16 operands, fp32 accumulate (fast mode) */
#define ONNXB200_PREC_FP32 3        /* CUDA-core fp32 FFMA (exactness reference on device) */

#define ONNXB200_LAYOUT_NCHW 0
#define ONNXB200_LAYOUT_NHWC 1

/* Conv auto_pad (src/ops/nn/conv.rs AutoPadding) */
#define ONNXB200_AUTOPAD_NOTSET 0
#define ONNXB200_AUTOPAD_SAME_UPPER 1
#define ONNXB200_AUTOPAD_SAME_LOWER 2
#define ONNXB200_AUTOPAD_VALID 3

/* Epilogue flags: what is fused after the contraction. */
#define ONNXB200_EPI_BIAS 1     /* + bias[C_out] (Conv input B / MatMul+Add bias) */
#define ONNXB200_EPI_BN 2       /* BatchNormalization (inference) folded to scale/shift */
#define ONNXB200_EPI_RESIDUAL 4 /* + residual tensor, same shape as the output (Add) */
#define ONNXB200_EPI_RELU 8     /* Relu (v > 0 ? v : 0) */

/* ---------------------------------------------------------------- handle */
typedef struct onnxb200_options {
  int precision;          /* ONNXB200_PREC_*; default 3XTF32 */
  size_t workspace_bytes; /* stream-ordered scratch; 0 = 64 MiB, the reference's
                             default workspace (src/execution/context.rs:63-82) */
  int use_cuda_graph;     /* graph runs are captured once and replayed (default 1) */
  int wait_timeout_ms;    /* host-side bound of onnxb200_synchronize (default 60000) */
} onnxb200_options;

typedef struct onnxb200_handle onnxb200_handle;

/* Library version (major*10000 + minor*100 + patch). */
ONNXB200_API int onnxb200_version(void);
/* Fills the defaults listed in onnxb200_options. */
ONNXB200_API void onnxb200_default_options(onnxb200_options* opts);
/* Creates a handle on `device` (replaces ExecutionContext::new + its workspace,
 * src/execution/context.rs:285-400).  opts may be NULL. */
ONNXB200_API int onnxb200_create(int device, const onnxb200_options* opts, onnxb200_handle** out);
ONNXB200_API int onnxb200_destroy(onnxb200_handle* h);
/* Message of the last failure on this handle ("" if none).  Valid until the next call. */
ONNXB200_API const char* onnxb200_last_error(const onnxb200_handle* h);
/* Message for a status code. */
ONNXB200_API const char* onnxb200_status_string(int status);
/* Runs subsequent work on a caller-owned cudaStream_t (NULL = the handle's own
 * stream, a blocking stream ordered with the legacy default stream). */
ONNXB200_API int onnxb200_set_stream(onnxb200_handle* h, void* cuda_stream);
ONNXB200_API void* onnxb200_get_stream(onnxb200_handle* h);
/* Waits for the handle's stream (bounded) and checks the device status word. */
ONNXB200_API int onnxb200_synchronize(onnxb200_handle* h);
/* Number of kernels this library launched on the handle since creation. */
ONNXB200_API int64_t onnxb200_kernel_launches(const onnxb200_handle* h);
/* Number of SMs of the handle's device. */
ONNXB200_API int onnxb200_num_sms(const onnxb200_handle* h);
/* Device memory on the handle's GPU, for bindings without a CUDA runtime of
 * their own (the reference's operators take host tensors: copy in, compute,
 * copy out).  Copies are asynchronous on the handle's stream (synchronize
 * before reading a device-to-host copy's destination). */
#define ONNXB200_COPY_H2D 0
#define ONNXB200_COPY_D2H 1
#define ONNXB200_COPY_D2D 2
ONNXB200_API int onnxb200_malloc(onnxb200_handle* h, size_t bytes, void** ptr);
ONNXB200_API int onnxb200_free(onnxb200_handle* h, void* ptr);
ONNXB200_API int onnxb200_memcpy(onnxb200_handle* h, void* dst, const void* src, size_t bytes, int kind);

/* ---------------------------------------------------------------- Conv */
typedef struct onnxb200_conv_desc {
  int64_t n, c, h, w;         /* input dims (logical NCHW) */
  int64_t c_out, kh, kw;      /* weight dims OIHW: [c_out, c/group, kh, kw] */
  int64_t stride_h, stride_w; /* default 1 */
  int64_t pad_top, pad_left, pad_bottom, pad_right;
  int64_t dil_h, dil_w;       /* default 1 */
  int64_t group;              /* default 1 */
  int auto_pad;               /* ONNXB200_AUTOPAD_* */
  int layout;                 /* layout of x, residual and y */
  int epilogue;               /* ONNXB200_EPI_* */
  int precision;              /* ONNXB200_PREC_* or DEFAULT */
  float bn_epsilon;           /* BatchNormalization epsilon (default 1e-5) */
} onnxb200_conv_desc;

/* Conv::output_shapes (src/ops/nn/conv.rs:205-323): out[4] = N, C_out, OH, OW. */
ONNXB200_API int onnxb200_conv2d_output_shape(const onnxb200_conv_desc* d, int64_t out[4]);

/* 1-D, 2-D and 3-D Conv (compute_conv, src/ops/nn/conv.rs:534-606; spatial
 * dims of 1-D in[0] = L, of 2-D in = {H, W}, of 3-D in = {D, H, W}, likewise the
 * other arrays).  x / y are NCL, NCHW or NCDHW; w is [c_out][c/group][k...];
 * bias [c_out] or NULL; relu != 0 fuses Relu.  1-D runs as a 2-D convolution of
 * height 1 on the tensor-core path (the handle's precision); 3-D runs on CUDA
 * cores in fp32 (compute_conv3d_direct_impl, conv.rs:938-1038). */
typedef struct onnxb200_conv_nd_desc {
  int spatial;                 /* 1, 2 or 3 */
  int64_t n, c, c_out, group;  /* group 0 = 1 */
  int64_t in[3], kernel[3];
  int64_t stride[3];           /* 0 = 1 */
  int64_t pad_begin[3], pad_end[3];
  int64_t dilation[3];         /* 0 = 1 */
  int auto_pad;                /* ONNXB200_AUTOPAD_* */
  int relu;
} onnxb200_conv_nd_desc;
/* Conv::output_shapes (conv.rs:205-323) for 1 to 3 spatial dims: out[0..rank). */
ONNXB200_API int onnxb200_conv_nd_output_shape(const onnxb200_conv_nd_desc* d, int64_t out[5], int* rank);
ONNXB200_API int onnxb200_conv_nd(onnxb200_handle* h, const onnxb200_conv_nd_desc* d, const float* x,
                                  const float* w, const float* bias, float* y);

/* Conv::compute (src/ops/nn/conv.rs:156-203 -> compute_conv :534-606) with the
 * optional fused epilogue.  w is OIHW; bias [c_out] if EPI_BIAS; bn_* [c_out]
 * (ONNX scale, B, mean, var) if EPI_BN; residual shaped like y if EPI_RESIDUAL.
 * Packs the weights into the handle's workspace on every call; use a conv plan
 * to pack once. */
ONNXB200_API int onnxb200_conv2d(onnxb200_handle* h, const onnxb200_conv_desc* d, const float* x,
                                 const float* w, const float* bias, const float* bn_scale,
                                 const float* bn_bias, const float* bn_mean, const float* bn_var,
                                 const float* residual, float* y);

/* Prepared convolution: weights packed (NHWC K-order, tf32 hi/lo split or bf16)
 * and BN folded once, at load time -- the layout change the reference's
 * TensorLayout (src/layout/tensor_layout.rs:8-513) does not have. */
typedef struct onnxb200_conv_plan onnxb200_conv_plan;
ONNXB200_API int onnxb200_conv_plan_create(onnxb200_handle* h, const onnxb200_conv_desc* d,
                                           const float* w, const float* bias,
                                           const float* bn_scale, const float* bn_bias,
                                           const float* bn_mean, const float* bn_var,
                                           onnxb200_conv_plan** out);
ONNXB200_API int onnxb200_conv_plan_run(onnxb200_handle* h, const onnxb200_conv_plan* p,
                                        const float* x, const float* residual, float* y);
ONNXB200_API int onnxb200_conv_plan_destroy(onnxb200_conv_plan* p);

/* Conv2d + fused epilogue on NHWC device buffers that allocates no device
 * memory.  No counterpart in the reference: it exists for callers that cannot
 * call cudaMalloc while they run (a host framework that owns all device memory
 * and hands in pre-sized input/output buffers, or a serving loop that cannot
 * take an allocation or the synchronisation of a cudaFree).  Instead of a
 * handle's growable workspace it uses one fixed array of
 * ONNXB200_NOALLOC_SCRATCH_BYTES in device memory, defined in the library and
 * held by every GPU that loads the library until the process exits; packed
 * weights + epilogue vectors larger than that are rejected with
 * ONNXB200_ERR_RESOURCE_EXHAUSTED (every ResNet-18/50 convolution fits).
 * Runs on the current device and the given stream (NULL = legacy default
 * stream) and blocks until y is written (bounded wait); device-side failures
 * are returned as status codes.  Because it blocks, it returns
 * ONNXB200_ERR_UNSUPPORTED on a stream that is being captured.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress).  All
 * calls share the array: calls that overlap on the GPU (e.g. issued
 * concurrently from several host threads) race on it.  If a call returns
 * ONNXB200_ERR_TIMEOUT its kernels may still be running; the next call on the
 * device first waits (bounded) for them before it reuses the array.
 * d->layout must be ONNXB200_LAYOUT_NHWC. */
#define ONNXB200_NOALLOC_SCRATCH_BYTES (24u << 20)
ONNXB200_API int onnxb200_conv2d_nhwc_noalloc(void* cuda_stream, const onnxb200_conv_desc* d,
                                              const float* x, const float* w, const float* bias,
                                              const float* bn_scale, const float* bn_bias,
                                              const float* bn_mean, const float* bn_var,
                                              const float* residual, float* y);

/* ---------------------------------------------------------------- MatMul / Gemm */
/* validate_matmul_shapes (src/ops/math/matmul.rs:401-487).  out_shape holds
 * max(a_rank, b_rank) entries. */
ONNXB200_API int onnxb200_matmul_output_shape(const int64_t* a_shape, int a_rank,
                                              const int64_t* b_shape, int b_rank,
                                              int64_t* out_shape, int* out_rank);
/* compute_matmul (src/ops/math/matmul.rs:124-279): numpy-broadcast batched
 * MatMul, row-major.  bias [N] (may be NULL) and EPI_RELU in `flags` fuse the
 * MatMul+Add(+Relu) pattern of the fusion pass (src/optimization/passes/fusion.rs:227-288). */
ONNXB200_API int onnxb200_matmul(onnxb200_handle* h, const float* a, const int64_t* a_shape,
                                 int a_rank, const float* b, const int64_t* b_shape, int b_rank,
                                 const float* bias, int flags, int precision, float* y);
/* Gemm::compute / compute_gemm (src/ops/math/gemm.rs:17-44, :172-291) with ONNX
 * attributes honoured: Y = alpha*op(A)*op(B) + beta*C, C (may be NULL)
 * unidirectionally broadcast from c_shape (rank 0..2) to [M, N]. */
ONNXB200_API int onnxb200_gemm(onnxb200_handle* h, const float* a, const float* b, const float* c,
                               const int64_t* c_shape, int c_rank, int64_t m, int64_t n,
                               int64_t k, int trans_a, int trans_b, float alpha, float beta,
                               int flags, int precision, float* y);

/* ---------------------------------------------------------------- pooling / elementwise */
/* MaxPool::compute / max_pool (src/ops/nn/pool.rs:168-193, :307-393) with
 * explicit ONNX attributes.  indices (may be NULL) receive int64 flat NCHW
 * indices of the first maximum (ONNX MaxPool output 1). out[4] gets the shape. */
ONNXB200_API int onnxb200_maxpool2d(onnxb200_handle* h, int layout, int64_t n, int64_t c,
                                    int64_t hh, int64_t ww, int64_t kh, int64_t kw,
                                    int64_t stride_h, int64_t stride_w, int64_t pad_top,
                                    int64_t pad_left, int64_t pad_bottom, int64_t pad_right,
                                    int ceil_mode, const float* x, float* y, int64_t* indices,
                                    int64_t out[4]);
/* GlobalAveragePool::compute / global_pool (src/ops/nn/pool.rs:275-295, :493-557). */
ONNXB200_API int onnxb200_global_avgpool(onnxb200_handle* h, int layout, int64_t n, int64_t c,
                                         int64_t hh, int64_t ww, const float* x, float* y);
/* element_wise_binary_op(+) with broadcasting (src/ops/tensor.rs:1124-1218); relu != 0 fuses Relu. */
ONNXB200_API int onnxb200_add(onnxb200_handle* h, const float* a, const int64_t* a_shape,
                              int a_rank, const float* b, const int64_t* b_shape, int b_rank,
                              int relu, float* y);
/* relu (src/ops/activations.rs:244-246). */
ONNXB200_API int onnxb200_relu(onnxb200_handle* h, const float* x, int64_t count, float* y);
/* ONNX BatchNormalization (inference); the reference registers no such operator. */
ONNXB200_API int onnxb200_batchnorm(onnxb200_handle* h, int layout, int64_t n, int64_t c,
                                    int64_t hh, int64_t ww, const float* x, const float* scale,
                                    const float* bias, const float* mean, const float* var,
                                    float epsilon, float* y);
/* Layout repacks (src/layout/tensor_layout.rs has no NHWC; these add it).
 * c_pad >= c zero-fills extra channels. */
ONNXB200_API int onnxb200_nchw_to_nhwc(onnxb200_handle* h, int64_t n, int64_t c, int64_t hh,
                                       int64_t ww, int64_t c_pad, const float* x, float* y);
ONNXB200_API int onnxb200_nhwc_to_nchw(onnxb200_handle* h, int64_t n, int64_t c, int64_t hh,
                                       int64_t ww, const float* x, float* y);

/* ---------------------------------------------------------------- graphs */
/* ONNX-style node list (the reference IR's Node, src/model.rs:162-172). */
#define ONNXB200_ATTR_INT 0
#define ONNXB200_ATTR_FLOAT 1
#define ONNXB200_ATTR_INTS 2
#define ONNXB200_ATTR_STRING 3
typedef struct onnxb200_attr {
  const char* name;
  int type;            /* ONNXB200_ATTR_* */
  int64_t i;
  float f;
  const int64_t* ints;
  int n_ints;
  const char* s;
} onnxb200_attr;

typedef struct onnxb200_node {
  const char* op_type; /* Conv, BatchNormalization, Relu, Add, MaxPool,
                          GlobalAveragePool, Flatten, Gemm, MatMul */
  const char* const* inputs;
  int n_inputs;        /* empty string = absent optional input */
  const char* const* outputs;
  int n_outputs;
  const onnxb200_attr* attrs;
  int n_attrs;
} onnxb200_node;

/* Named tensor: initializer (data = HOST fp32) or graph input (data ignored). */
typedef struct onnxb200_tensor_info {
  const char* name;
  const float* data;
  const int64_t* shape;
  int rank;
} onnxb200_tensor_info;

typedef struct onnxb200_graph_stats {
  int n_nodes_in;        /* nodes given */
  int n_steps;           /* executable steps after fusion */
  int n_fused;           /* nodes absorbed into an epilogue */
  int64_t kernels_per_run; /* kernel launches per onnxb200_graph_run */
  int64_t arena_bytes;   /* activation arena (planned, one allocation) */
  int64_t weight_bytes;  /* packed weights */
  int captured;          /* 1 if runs replay a CUDA graph */
  int bf16_tensors;      /* activations stored as bf16 (BF16 precision) */
} onnxb200_graph_stats;

typedef struct onnxb200_graph onnxb200_graph;

/* ExecutionEngine::prepare (src/execution/engine.rs:110-163): fusion (Conv +
 * BatchNormalization [+ residual Add] [+ Relu], MatMul + Add [+ Relu]),
 * weight packing, static memory plan of all activations in one device arena
 * (first-fit over lifetimes, src/memory/planner.rs:2428-2498, :3554-3750). */
ONNXB200_API int onnxb200_graph_build(onnxb200_handle* h, const onnxb200_node* nodes, int n_nodes,
                                      const onnxb200_tensor_info* initializers, int n_init,
                                      const onnxb200_tensor_info* inputs, int n_inputs,
                                      const char* const* outputs, int n_outputs,
                                      onnxb200_graph** out);
/* ExecutionEngine::run (src/execution/engine.rs:166-231) on device buffers
 * (NCHW, shapes as built).  Asynchronous on the handle's stream; the first run
 * captures a CUDA graph when use_cuda_graph is set. */
ONNXB200_API int onnxb200_graph_run(onnxb200_handle* h, onnxb200_graph* g,
                                    const float* const* inputs, float* const* outputs);
/* Same, from and to HOST buffers: copies in, runs, copies out, synchronizes. */
ONNXB200_API int onnxb200_graph_run_host(onnxb200_handle* h, onnxb200_graph* g,
                                         const float* const* inputs, float* const* outputs);
/* A sequence of n_batches host batches (inputs[b * n_inputs + i], outputs
 * [b * n_outputs + i]; pinned host memory for the copies to overlap): batch b+1's
 * host-to-device input copy runs on a copy stream as soon as batch b's graph has
 * read its inputs, overlapping the rest of batch b.  Synchronizes at the end.
 * The serving counterpart of calling ExecutionEngine::run once per batch
 * (src/execution/engine.rs:166-231). */
ONNXB200_API int onnxb200_graph_run_host_pipelined(onnxb200_handle* h, onnxb200_graph* g,
                                                   int n_batches, const float* const* inputs,
                                                   float* const* outputs);
ONNXB200_API int onnxb200_graph_output_shape(const onnxb200_graph* g, int index, int64_t* shape,
                                             int* rank);

/* Shape inference over a whole node list without building a graph: host only
 * (no handle, no GPU, no device memory).  The planner's
 * infer_node_output_shapes (src/memory/planner.rs:908-960), i.e.
 * Operator::output_shapes (src/ops/registry.rs:14-27) applied node by node in
 * topological order.  `known` gives the shapes of the initializers and graph
 * inputs (their data is not read and may be NULL).  Fills shapes[0..max_shapes)
 * with every node output, node by node in the given order (name points into
 * `nodes`); *n_shapes receives the count, and ONNXB200_ERR_RESOURCE_EXHAUSTED
 * is returned when it exceeds max_shapes.  Errors as onnxb200_graph_build
 * (ValidationError for inconsistent shapes, InvalidOperator for an op that is
 * not on this path, InvalidGraph for a cycle or a tensor without a producer);
 * the message goes to err (may be NULL). */
typedef struct onnxb200_shape_info {
  const char* name;
  int64_t dims[8];
  int rank;
} onnxb200_shape_info;
ONNXB200_API int onnxb200_infer_shapes(const onnxb200_node* nodes, int n_nodes,
                                       const onnxb200_tensor_info* known, int n_known,
                                       onnxb200_shape_info* shapes, int max_shapes, int* n_shapes,
                                       char* err, size_t err_len);

/* Per-step profile of one eager run: the device-side counterpart of the
 * reference's per-node profiling events (src/execution/engine.rs:549-649,
 * src/tools/profiler/core.rs:726-791). */
#define ONNXB200_STEP_CONV_TC 1     /* tcgen05 implicit-GEMM convolution */
#define ONNXB200_STEP_CONV_DIRECT 2 /* CUDA-core convolution (grouped / fp32 mode) */
#define ONNXB200_STEP_GEMM 3        /* Gemm / MatMul on the tcgen05 GEMM core */
#define ONNXB200_STEP_MAXPOOL 4
#define ONNXB200_STEP_GAP 5
#define ONNXB200_STEP_ADD 6
#define ONNXB200_STEP_RELU 7
#define ONNXB200_STEP_AFFINE 8      /* standalone BatchNormalization */
#define ONNXB200_STEP_CONVERT 9     /* layout conversion / copy at the graph edges */
typedef struct onnxb200_step_profile {
  int kind;      /* ONNXB200_STEP_* */
  float ms;      /* device time (CUDA events around the step) */
  double flops;  /* algorithmic FLOPs (2*M*N*K for contractions, 0 otherwise) */
  double bytes;  /* algorithmic bytes: each input read once, the output written once */
} onnxb200_step_profile;
ONNXB200_API int onnxb200_graph_profile(onnxb200_handle* h, onnxb200_graph* g,
                                        const float* const* inputs, float* const* outputs,
                                        onnxb200_step_profile* steps, int max_steps, int* n_steps);
ONNXB200_API int onnxb200_graph_get_stats(const onnxb200_graph* g, onnxb200_graph_stats* st);
ONNXB200_API int onnxb200_graph_destroy(onnxb200_graph* g);

/* ---------------------------------------------------------------- several GPUs */
/* Batch-sharded replicas of one graph on several GPUs of this process, for a
 * host that drives all of them from one process (one process per GPU can
 * instead build one graph per process on its own slice).  Every graph input is
 * split along its first dimension into contiguous slices, one per device (the
 * first batch % n_devices devices take one image more); each device holds a full
 * copy of the packed weights; there is no collective.  The reference runs one
 * graph on host cores (ExecutionEngine::run_concurrent,
 * src/execution/engine.rs:743-809) and has no multi-device path.
 * inputs[] carry the FULL batch shapes; every output must have the batch as its
 * first dimension.  opts as for onnxb200_create (NULL = defaults).  Builds the
 * devices in parallel, one host thread each. */
typedef struct onnxb200_multi onnxb200_multi;
ONNXB200_API int onnxb200_multi_build(const int* devices, int n_devices, const onnxb200_options* opts,
                                      const onnxb200_node* nodes, int n_nodes,
                                      const onnxb200_tensor_info* initializers, int n_init,
                                      const onnxb200_tensor_info* inputs, int n_inputs,
                                      const char* const* outputs, int n_outputs, onnxb200_multi** out,
                                      char* err, size_t err_len);
/* Runs n_batches full batches from HOST buffers (inputs[b * n_inputs + i],
 * outputs[b * n_outputs + o]; pinned memory lets the copies overlap): one host
 * thread per device copies its rows of each input in, replays its graph
 * (onnxb200_graph_run_host_pipelined) and copies its rows of each output into
 * the disjoint rows of the caller's output buffers.  The threads start together
 * from a host barrier; each device's time from that release to its last
 * completion event is kept for onnxb200_multi_get_info.  Returns when every
 * device is done (bounded waits as onnxb200_synchronize). */
ONNXB200_API int onnxb200_multi_run_host(onnxb200_multi* m, int n_batches, const float* const* inputs,
                                         float* const* outputs);
/* n_devices, batch, slice_begin[n_devices] (first image of each device's slice)
 * and last_run_ms[n_devices] (the last run's device time per device); any
 * pointer may be NULL. */
ONNXB200_API int onnxb200_multi_get_info(const onnxb200_multi* m, int* n_devices, int64_t* batch,
                                         int64_t* slice_begin, float* last_run_ms);
/* Full-batch shape of output `index`. */
ONNXB200_API int onnxb200_multi_output_shape(const onnxb200_multi* m, int index, int64_t* shape, int* rank);
/* Message of the last failed run ("" if none). */
ONNXB200_API const char* onnxb200_multi_last_error(const onnxb200_multi* m);
ONNXB200_API int onnxb200_multi_destroy(onnxb200_multi* m);

/* ---------------------------------------------------------------- ONNX models */
/* A parsed .onnx ModelProto, host memory only (no handle, no GPU needed):
 * OnnxModelLoader (src/parser/model_loader.rs:27-454) restricted to the main
 * graph -- nodes with INT / FLOAT / STRING / INTS attributes (others are counted
 * and skipped), fp32 initializers (inline raw_data / float_data, or external
 * data next to the model file; other element types are counted and skipped),
 * graph inputs that are not initializers (symbolic dimensions read as -1) and
 * graph outputs.  Errors: ONNXB200_ERR_PROTOBUF (malformed bytes),
 * ONNXB200_ERR_INVALID_MODEL (no graph, undefined attribute type, a value
 * without a type, data that does not match its shape), ONNXB200_ERR_IO,
 * ONNXB200_ERR_UNSUPPORTED (segmented tensors; external data when parsing
 * from memory without base_dir); the message goes to err (may be NULL). */
typedef struct onnxb200_model onnxb200_model;
typedef struct onnxb200_model_info {
  int64_t ir_version;
  int64_t opset;                  /* version imported for the default domain (1 if none) */
  int n_nodes;
  int n_initializers;             /* fp32 initializers */
  int n_skipped_initializers;     /* initializers of other element types */
  int n_skipped_attributes;       /* attributes with no onnxb200_attr form */
  int n_inputs;                   /* graph inputs that are not initializers */
  int n_outputs;
  const char* producer_name;
  const char* graph_name;
} onnxb200_model_info;
/* OnnxModelLoader::load_model_from_bytes (model_loader.rs:40-43); base_dir
 * (may be NULL) is where external data files are looked up. */
ONNXB200_API int onnxb200_model_parse(const void* data, size_t len, const char* base_dir,
                                      onnxb200_model** out, char* err, size_t err_len);
/* OnnxModelLoader::load_model (model_loader.rs:27-37). */
ONNXB200_API int onnxb200_model_load(const char* path, onnxb200_model** out, char* err, size_t err_len);
ONNXB200_API int onnxb200_model_get_info(const onnxb200_model* m, onnxb200_model_info* info);
/* Views into the model (valid until onnxb200_model_destroy), in the forms
 * onnxb200_graph_build takes. */
ONNXB200_API int onnxb200_model_get_nodes(const onnxb200_model* m, const onnxb200_node** nodes, int* n);
ONNXB200_API int onnxb200_model_get_initializers(const onnxb200_model* m, const onnxb200_tensor_info** t,
                                                 int* n);
ONNXB200_API int onnxb200_model_get_inputs(const onnxb200_model* m, const onnxb200_tensor_info** t, int* n);
ONNXB200_API int onnxb200_model_get_outputs(const onnxb200_model* m, const char* const** names, int* n);
ONNXB200_API int onnxb200_model_destroy(onnxb200_model* m);
/* onnxb200_graph_build over a parsed model; input_shapes (matched by name)
 * replace the model's input shapes, which must then all be concrete. */
ONNXB200_API int onnxb200_graph_build_from_model(onnxb200_handle* h, const onnxb200_model* m,
                                                 const onnxb200_tensor_info* input_shapes,
                                                 int n_input_shapes, onnxb200_graph** out);

#ifdef __cplusplus
}
#endif
#endif /* ONNXB200_H */
