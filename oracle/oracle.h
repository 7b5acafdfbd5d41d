/*
 * CPU oracle for the onnx-rs Conv / MatMul / Gemm / pool / elementwise hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference's
 * CPU operators (aslitaser/onnx-rs, Rust).  Only the test-suite, the smoke check
 * and the CPU-baseline leg of bench.py load it, and only as the checker or as the
 * timed CPU baseline.  The product library (libonnxb200.so) never links or calls it.
 *
 * All tensors are fp32, row-major, NCHW for activations and OIHW for conv
 * weights, exactly like the reference's `Tensor { data: ArrayD<f32> }`
 * (src/ops/tensor.rs:206-218).
 *
 * Accumulation modes (the `acc64` argument):
 *   0 = reference-faithful: fp32 accumulators, summation over K in the same
 *       order as the reference loops (ic, kh, kw) / (k).
 *   1 = diagnostic: fp64 accumulators, rounded to fp32 once at the end.
 *
 * Parity pins: conv1d/conv2d/conv3d/grouped/padding known answers from
 * src/ops/nn/conv.rs:1487-1768 and the correct MatMul cases from
 * src/ops/math/matmul.rs:747-795 are reproduced bit-exactly by this code
 * (tests/test_oracle.py against tests/golden/).  Pool, Gemm attributes, Add,
 * BatchNormalization and Flatten have no reference tests: they follow the
 * reference code (pool.rs, tensor.rs) or, where the reference has no operator,
 * the ONNX operator specification.
 */
#ifndef ONNXB200_ORACLE_H
#define ONNXB200_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORC_OK = 0,
  ORC_ERR_VALIDATION = 1, /* reference Error::ValidationError */
  ORC_ERR_UNSUPPORTED = 2 /* reference Error::UnsupportedFeature */
};

/* Strategies of src/ops/nn/conv.rs:1399-1459 (Auto resolves like the reference). */
enum { ORC_CONV_AUTO = 0, ORC_CONV_DIRECT = 1, ORC_CONV_IM2COL = 2, ORC_CONV_SIMD = 3 };

/* Output size of one spatial dim (conv.rs:319-320, planner.rs infer_conv_shape). */
int64_t orc_conv_out_dim(int64_t in, int64_t k, int64_t stride, int64_t pad_head,
                         int64_t pad_tail, int64_t dilation);

/* SAME_UPPER (mode 1) / SAME_LOWER (mode 2) padding split (conv.rs:426-458). */
void orc_same_pads(int64_t in, int64_t k, int64_t stride, int64_t dilation, int mode,
                   int64_t* pad_head, int64_t* pad_tail);

/* Which strategy the reference's Auto mode picks (conv.rs:1399-1459), 2-D only. */
int orc_conv_strategy(int64_t kh, int64_t kw, int64_t group);

/* 2-D convolution, NCHW x OIHW -> NCHW.  bias may be NULL. */
int orc_conv2d(const float* x, int64_t n, int64_t c, int64_t h, int64_t w,
               const float* wt, int64_t co, int64_t kh, int64_t kw, const float* bias,
               int64_t sh, int64_t sw, int64_t pt, int64_t pl, int64_t pb, int64_t pr,
               int64_t dh, int64_t dw, int64_t group, int strategy, int acc64,
               int nthreads, float* y);

/* N-d direct convolution for 1-D and 3-D known answers (conv.rs:609-706). */
int orc_conv_nd_direct(const float* x, const int64_t* xshape, int rank, const float* wt,
                       const int64_t* wshape, const float* bias, const int64_t* strides,
                       const int64_t* pads, const int64_t* dilations, int64_t group,
                       float* y, int64_t* yshape);

/* numpy-broadcast MatMul (matmul.rs:124-279, validate :401-487).  out_shape must
 * hold max(ra, rb) entries; *out_rank receives the output rank. */
int orc_matmul_shape(const int64_t* as, int ra, const int64_t* bs, int rb,
                     int64_t* out_shape, int* out_rank);
int orc_matmul(const float* a, const int64_t* as, int ra, const float* b,
               const int64_t* bs, int rb, int acc64, int nthreads, float* y);

/* ONNX Gemm: Y = alpha*op(A)*op(B) + beta*C, C unidirectionally broadcast to
 * [M,N] (c_rank 0..2; c may be NULL).  compute_gemm (gemm.rs:172-291) with the
 * attributes honoured as the ONNX specification states. */
int orc_gemm(const float* a, const float* b, const float* c, const int64_t* cs,
             int c_rank, int64_t m, int64_t nn, int64_t k, int trans_a, int trans_b,
             float alpha, float beta, int acc64, float* y);

/* MaxPool 2-D (pool.rs:307-393): window max over in-bounds taps, init f32::MIN.
 * indices (may be NULL) receive the ONNX flat NCHW index of the first maximum. */
int orc_maxpool2d(const float* x, int64_t n, int64_t c, int64_t h, int64_t w,
                  int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t pt, int64_t pl,
                  int64_t pb, int64_t pr, int ceil_mode, float* y, int64_t* indices);

/* GlobalAveragePool (pool.rs:493-557): sequential fp32 sum / count. */
int orc_global_avgpool(const float* x, int64_t n, int64_t c, int64_t spatial, float* y);

/* Relu (activations.rs:244-246): v > 0 ? v : 0. */
void orc_relu(const float* x, int64_t count, float* y);

/* Broadcast Add (tensor.rs:1124-1218 with get_broadcast_shape :1536-1571). */
int orc_broadcast_shape(const int64_t* as, int ra, const int64_t* bs, int rb,
                        int64_t* out_shape, int* out_rank);
int orc_add(const float* a, const int64_t* as, int ra, const float* b, const int64_t* bs,
            int rb, float* y);

/* ONNX BatchNormalization (inference): y = (x - mean) / sqrt(var + eps) * scale + B. */
int orc_batchnorm(const float* x, int64_t n, int64_t c, int64_t spatial, const float* scale,
                  const float* bias, const float* mean, const float* var, float eps, float* y);

#ifdef __cplusplus
}
#endif
#endif
