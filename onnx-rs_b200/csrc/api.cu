// C-ABI implementation: handle, workspace, TMA maps, Conv plans, MatMul, Gemm,
// pooling, elementwise and layout entry points of include/onnxb200.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "internal.h"

using namespace ob2;

namespace ob2 {

namespace {
constexpr size_t kAlign = 256;
inline size_t align_up(size_t v, size_t a = kAlign) { return (v + a - 1) / a * a; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
}  // namespace

int set_error(onnxb200_handle* h, int code, const std::string& msg) {
  if (h) h->last_error = msg;
  return code;
}

int cuda_check(onnxb200_handle* h, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ONNXB200_OK;
  return set_error(h, e == cudaErrorMemoryAllocation ? ONNXB200_ERR_RESOURCE_EXHAUSTED
                                                     : ONNXB200_ERR_EXECUTION,
                   std::string(what) + ": " + cudaGetErrorString(e));
}

int ensure_workspace(onnxb200_handle* h, size_t bytes) {
  if (bytes <= h->ws_bytes) return ONNXB200_OK;
  // Grow: wait for in-flight users of the old buffer, then replace it.
  cudaError_t e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return cuda_check(h, e, "workspace sync");
  if (h->ws) cudaFree(h->ws);
  h->ws = nullptr;
  h->ws_bytes = 0;
  size_t nb = std::max(align_up(bytes, 1 << 20), h->opts.workspace_bytes);
  e = cudaMalloc(&h->ws, nb);
  if (e != cudaSuccess) return cuda_check(h, e, "workspace allocation");
  h->ws_bytes = nb;
  return ONNXB200_OK;
}

int encode_weight_map(onnxb200_handle* h, CUtensorMap* map, const void* base, int rows, int kpad,
                      int prec, int bn, int bk) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(h, ONNXB200_ERR_EXECUTION, "cuTensorMapEncodeTiled unavailable");
  const int esz = prec == kPrecBF16 ? 2 : 4;
  cuuint64_t dims[2] = {(cuuint64_t)kpad, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kpad * esz};
  // one k-block of a weight row = bk elements: 128 bytes of fp32 or (bk = 64)
  // of bf16 (128-byte swizzle), or 64 bytes of bf16 (bk = 32, 64-byte swizzle)
  cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)bn};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, prec == kPrecBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                  2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  bk * esz == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(h, ONNXB200_ERR_EXECUTION, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return ONNXB200_OK;
}

static int64_t conv_out_dim(int64_t in, int64_t k, int64_t s, int64_t ph, int64_t pt, int64_t d) {
  const int64_t dk = (k - 1) * d + 1;
  const int64_t span = in + ph + pt - dk;
  if (span < 0) return 0;
  return span / s + 1;
}

int resolve_conv_desc(onnxb200_handle* h, const onnxb200_conv_desc* in, onnxb200_conv_desc* o,
                      int64_t* oh, int64_t* ow) {
  if (!in) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "null conv descriptor");
  *o = *in;
  if (o->stride_h <= 0) o->stride_h = 1;
  if (o->stride_w <= 0) o->stride_w = 1;
  if (o->dil_h <= 0) o->dil_h = 1;
  if (o->dil_w <= 0) o->dil_w = 1;
  if (o->group <= 0) o->group = 1;
  if (o->bn_epsilon <= 0.f) o->bn_epsilon = 1e-5f;
  if (o->n < 0 || o->c <= 0 || o->h <= 0 || o->w <= 0 || o->c_out <= 0 || o->kh <= 0 || o->kw <= 0)
    return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: non-positive dimension");
  // compute_conv_direct (src/ops/nn/conv.rs:628-644)
  if (o->c % o->group != 0 || o->c_out % o->group != 0)
    return set_error(h, ONNXB200_ERR_VALIDATION,
                     "Input and output channels must be divisible by groups");
  auto same = [&](int64_t inp, int64_t k, int64_t s, int64_t d, bool upper, int64_t* head,
                  int64_t* tail) {
    // calculate_same_padding (src/ops/nn/conv.rs:426-458)
    const int64_t dk = (k - 1) * d + 1;
    const int64_t out = (inp + s - 1) / s;
    const int64_t need = (out - 1) * s + dk - inp;
    *head = *tail = 0;
    if (need > 0) {
      if (upper) {
        *head = need / 2;
        *tail = need - *head;
      } else {
        *tail = need / 2;
        *head = need - *tail;
      }
    }
  };
  switch (o->auto_pad) {
    case ONNXB200_AUTOPAD_NOTSET:
      break;
    case ONNXB200_AUTOPAD_SAME_UPPER:
    case ONNXB200_AUTOPAD_SAME_LOWER: {
      const bool up = o->auto_pad == ONNXB200_AUTOPAD_SAME_UPPER;
      same(o->h, o->kh, o->stride_h, o->dil_h, up, &o->pad_top, &o->pad_bottom);
      same(o->w, o->kw, o->stride_w, o->dil_w, up, &o->pad_left, &o->pad_right);
      break;
    }
    case ONNXB200_AUTOPAD_VALID:
      o->pad_top = o->pad_left = o->pad_bottom = o->pad_right = 0;
      break;
    default:
      return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: unknown auto_pad");
  }
  o->auto_pad = ONNXB200_AUTOPAD_NOTSET;
  if (o->pad_top < 0 || o->pad_left < 0 || o->pad_bottom < 0 || o->pad_right < 0)
    return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: negative padding");
  *oh = conv_out_dim(o->h, o->kh, o->stride_h, o->pad_top, o->pad_bottom, o->dil_h);
  *ow = conv_out_dim(o->w, o->kw, o->stride_w, o->pad_left, o->pad_right, o->dil_w);
  if (*oh <= 0 || *ow <= 0)
    return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: kernel larger than padded input");
  if (o->layout != ONNXB200_LAYOUT_NCHW && o->layout != ONNXB200_LAYOUT_NHWC)
    return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: unknown layout");
  const int prec = resolve_prec(h, o->precision);
  if (prec < 0 || prec > 3) return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: unknown precision");
  o->precision = prec;
  if (o->n * o->c * o->h * o->w > (int64_t)INT32_MAX ||
      o->n * o->c_out * (*oh) * (*ow) > (int64_t)INT32_MAX * 4)
    return set_error(h, ONNXB200_ERR_UNSUPPORTED, "Conv: tensor too large");
  return ONNXB200_OK;
}

// Tile width and K split of a tensor-core plan (p->d, num_kb, a_bf16 set):
// K splits for fp32-activation problems with too few output tiles.
static void choose_tiling(onnxb200_handle* h, onnxb200_conv_plan* p, bool residual) {
  IgemmParams q{};
  q.M = (int)(p->d.n * p->oh * p->ow);
  q.Nc = (int)p->d.c_out;
  q.batches = 1;
  q.num_kb = p->num_kb;
  q.a_bf16 = p->a_bf16;
  q.out_bf16 = p->out_bf16;
  int bn = 128, ks = 1, smt = 0;
  igemm_pick_split(q, residual, p->prec, h->num_sms, &bn, &ks, &smt);
  p->bn = bn;
  p->ksplit = ks;
  p->split_mt = smt;
  p->split_bytes = ks > 1 ? (size_t)ks * (q.M - smt * 128) * q.Nc * sizeof(float) : 0;
}

void conv_plan_free(onnxb200_conv_plan* p) {
  (void)p;
}

int conv_plan_init(onnxb200_handle* h, const onnxb200_conv_desc* din, int cs_in, const float* w,
                   const float* bias, const float* bn_scale, const float* bn_bias,
                   const float* bn_mean, const float* bn_var, onnxb200_conv_plan* p, void* scratch,
                   size_t scratch_bytes, size_t* scratch_used, bool a_bf16, bool out_bf16) {
  int rc = resolve_conv_desc(h, din, &p->d, &p->oh, &p->ow);
  if (rc) return rc;
  const onnxb200_conv_desc& d = p->d;
  if (!w) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null weights");
  const bool want_bias = (d.epilogue & ONNXB200_EPI_BIAS) != 0;
  const bool want_bn = (d.epilogue & ONNXB200_EPI_BN) != 0;
  if (want_bias && !bias) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null bias");
  if (want_bn && (!bn_scale || !bn_bias || !bn_mean || !bn_var))
    return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null BatchNormalization parameter");
  p->prec = d.precision;
  p->cs_in = cs_in;
  p->use_tc = d.group == 1 && p->prec != kPrecFP32 && d.c_out % 4 == 0 && cs_in % 4 == 0 &&
              d.kh * d.kw * cs_in < (1 << 30);
  if ((a_bf16 || out_bf16) && (!p->use_tc || p->prec != kPrecBF16 || (a_bf16 && cs_in % 64)))
    return set_error(h, ONNXB200_ERR_UNSUPPORTED, "Conv: bf16 storage needs the BF16 tensor-core path");
  p->a_bf16 = a_bf16;
  p->out_bf16 = out_bf16;
  const int CO = (int)d.c_out;
  size_t need = 0;
  size_t off_hi = 0, off_lo = 0, off_scale = 0, off_shift = 0, off_w = 0, off_split = 0;
  p->pairs = p->use_tc && !a_bf16 && cs_in == 4 && d.stride_w == 2 && d.dil_w == 1 &&
             d.w % 2 == 0 && d.kw > 1;
  const int kwp = (int)((d.kw + (d.pad_left & 1) + 1) / 2);  // pair taps
  if (p->use_tc) {
    p->K = p->pairs ? (int)(d.kh * kwp * 8) : (int)(d.kh * d.kw * cs_in);
    p->kpad = igemm_kpad(p->K, p->prec, a_bf16);
    p->num_kb = p->kpad / igemm_block_k(p->prec, a_bf16);
    choose_tiling(h, p, (d.epilogue & ONNXB200_EPI_RESIDUAL) != 0);
    const size_t esz = p->prec == kPrecBF16 ? 2 : 4;
    const size_t wbytes = align_up((size_t)CO * p->kpad * esz);
    off_hi = need;
    need += wbytes;
    if (p->prec == kPrec3xTF32) {
      off_lo = need;
      need += wbytes;
    }
    p->weight_bytes = (int64_t)need;
    if (!scratch && !scratch_used && p->split_bytes) {  // op-level plans own their K-split buffer
      off_split = need;
      need += align_up(p->split_bytes);
    }
  } else {
    off_w = need;
    need += align_up((size_t)CO * (d.c / d.group) * d.kh * d.kw * sizeof(float));
    p->weight_bytes = (int64_t)need;
  }
  if (want_bn) {
    off_scale = need;
    need += align_up(CO * sizeof(float));
  }
  if (want_bn || want_bias) {
    off_shift = need;
    need += align_up(CO * sizeof(float));
  }
  uint8_t* basep = nullptr;
  if (!scratch && scratch_used) {  // size query only
    *scratch_used = need;
    return ONNXB200_OK;
  }
  if (scratch) {
    if (need > scratch_bytes)
      return set_error(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "Conv: scratch too small for packed weights");
    basep = static_cast<uint8_t*>(scratch);
    if (scratch_used) *scratch_used = need;
  } else {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&basep), need);
    if (e != cudaSuccess) return cuda_check(h, e, "conv plan allocation");
  }
  p->w_hi = p->w_lo = nullptr;
  p->w_oihw = nullptr;
  p->scale = p->shift = nullptr;
  cudaStream_t st = h->stream;
  p->split_ws = nullptr;
  if (p->use_tc) {
    p->w_hi = basep + off_hi;
    if (p->prec == kPrec3xTF32) p->w_lo = basep + off_lo;
    if (off_split) p->split_ws = reinterpret_cast<float*>(basep + off_split);
    // OIHW element (co, ci, r, s) -> k = (r*KW + s)*cs_in + ci
    rc = pack_b_launch(w, CO, p->K, p->kpad, cs_in, (int)d.c, CO, 0, d.c * d.kh * d.kw, 1,
                       d.kh * d.kw, p->prec, p->w_hi, p->w_lo, st, p->pairs ? (int)d.kw : 0,
                       (int)(d.pad_left & 1));
    h->launches++;
    if (rc) return cuda_check(h, (cudaError_t)rc, "weight packing");
    const int bk = igemm_block_k(p->prec, a_bf16);
    rc = encode_weight_map(h, &p->tm_hi, p->w_hi, CO, p->kpad, p->prec, p->bn, bk);
    if (rc) return rc;
    rc = encode_weight_map(h, &p->tm_lo, p->w_lo ? p->w_lo : p->w_hi, CO, p->kpad, p->prec, p->bn, bk);
    if (rc) return rc;
  } else {
    p->w_oihw = reinterpret_cast<float*>(basep + off_w);
    cudaError_t e = cudaMemcpyAsync(p->w_oihw, w, (size_t)CO * (d.c / d.group) * d.kh * d.kw * sizeof(float),
                                    cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_check(h, e, "weight copy");
  }
  if (want_bn) {
    p->scale = reinterpret_cast<float*>(basep + off_scale);
    p->shift = reinterpret_cast<float*>(basep + off_shift);
    rc = bn_fold_launch(bn_scale, bn_bias, bn_mean, bn_var, want_bias ? bias : nullptr, d.bn_epsilon,
                        CO, p->scale, p->shift, st);
    h->launches++;
    if (rc) return cuda_check(h, (cudaError_t)rc, "BatchNormalization fold");
  } else if (want_bias) {
    p->shift = reinterpret_cast<float*>(basep + off_shift);
    cudaError_t e = cudaMemcpyAsync(p->shift, bias, CO * sizeof(float), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_check(h, e, "bias copy");
  }
  return ONNXB200_OK;
}

int conv_plan_exec_nhwc(onnxb200_handle* h, const onnxb200_conv_plan* p, const float* x,
                        const float* residual, float* y, float* split_ws) {
  const onnxb200_conv_desc& d = p->d;
  const bool relu = (d.epilogue & ONNXB200_EPI_RELU) != 0;
  const float* res = (d.epilogue & ONNXB200_EPI_RESIDUAL) ? residual : nullptr;
  if ((d.epilogue & ONNXB200_EPI_RESIDUAL) && !residual)
    return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null residual");
  if (d.n == 0) return ONNXB200_OK;
  int rc;
  if (p->use_tc) {
    IgemmParams q{};
    q.x = x;
    q.Hin = (int)d.h;
    q.Win = (int)d.w;
    q.Cs = p->cs_in;
    q.OH = (int)p->oh;
    q.OW = (int)p->ow;
    q.KW = (int)d.kw;
    q.sh = (int)d.stride_h;
    q.sw = (int)d.stride_w;
    q.ph = (int)d.pad_top;
    q.pw = (int)d.pad_left;
    q.dh = (int)d.dil_h;
    q.dw = (int)d.dil_w;
    q.M = (int)(d.n * p->oh * p->ow);
    q.Nc = (int)d.c_out;
    q.K = p->K;
    q.num_kb = p->num_kb;
    q.batches = 1;
    q.y = y;
    q.ldy = (int)d.c_out;
    q.scale = p->scale;
    q.shift = p->shift;
    q.res = res;
    q.ldr = (int)d.c_out;
    q.relu = relu;
    q.status = h->d_status;
    q.m_tiles = (q.M + 127) / 128;
    q.n_tiles = (q.Nc + p->bn - 1) / p->bn;
    if (p->pairs) {  // the same NHWC memory as [N][H][W/2][8], stride 1 over pair taps
      q.Win = (int)(d.w / 2);
      q.Cs = 8;
      q.KW = (int)((d.kw + (d.pad_left & 1) + 1) / 2);
      q.sw = 1;
      q.pw = (int)((d.pad_left + 1) / 2);
    }
    q.a_bf16 = p->a_bf16;
    q.out_bf16 = p->out_bf16;
    q.a_mode = pick_a_mode(q, p->prec);
    CUtensorMap am{};
    if (q.a_mode != kALoadGather) {
      const int rows = q.a_mode == kALoadTma2d ? (int)d.n * q.Hin * q.Win : (int)d.n;
      const int er = encode_a_map(q, rows, &am);
      if (er) return set_error(h, ONNXB200_ERR_EXECUTION, "Conv: A tensor map encode failed: " + std::to_string(er));
    }
    float* ws = split_ws ? split_ws : p->split_ws;
    rc = igemm_launch_split(q, ws ? p->ksplit : 1, p->split_mt, ws, p->tm_hi, p->tm_lo, am, am, p->prec, p->bn,
                            h->num_sms, h->stream);
    if (ws && p->ksplit > 1) h->launches += p->split_mt > 0 ? 2 : 1;  // the reduction pass (and tail launch)
  } else {
    rc = conv_direct_launch(x, (int)d.n, (int)d.h, (int)d.w, (int)d.c, p->cs_in, p->w_oihw,
                            (int)d.c_out, (int)d.kh, (int)d.kw, (int)d.stride_h, (int)d.stride_w,
                            (int)d.pad_top, (int)d.pad_left, (int)d.dil_h, (int)d.dil_w,
                            (int)d.group, (int)p->oh, (int)p->ow, p->scale, p->shift, res, relu, y,
                            h->stream);
  }
  h->launches++;
  if (rc) return cuda_check(h, (cudaError_t)rc, "Conv launch");
  return ONNXB200_OK;
}

int conv_dual_plan_init(onnxb200_handle* h, const onnxb200_conv_desc* d1, int cs1, const float* w1,
                        const ConvBranchBN& bn1, const onnxb200_conv_desc* d2, int cs2, const float* w2,
                        const ConvBranchBN& bn2, onnxb200_conv_plan* p, void* scratch, size_t scratch_bytes,
                        size_t* scratch_used, bool a_bf16, bool out_bf16) {
  onnxb200_conv_desc r2;
  int64_t oh2 = 0, ow2 = 0;
  int rc = resolve_conv_desc(h, d1, &p->d, &p->oh, &p->ow);
  if (rc) return rc;
  rc = resolve_conv_desc(h, d2, &r2, &oh2, &ow2);
  if (rc) return rc;
  const onnxb200_conv_desc& a = p->d;
  if (!dual_conv_supported(a, cs1, r2, cs2) || oh2 != p->oh || ow2 != p->ow || a.precision != r2.precision)
    return set_error(h, ONNXB200_ERR_UNSUPPORTED, "Conv: these two convolutions cannot share one K loop");
  if (!w1 || !w2) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null weights");
  const int CO = (int)a.c_out;
  p->prec = a.precision;
  p->cs_in = cs1;
  p->use_tc = true;
  p->pairs = false;
  if ((a_bf16 || out_bf16) && (p->prec != kPrecBF16 || (a_bf16 && (a.c % 64 || r2.c % 64))))
    return set_error(h, ONNXB200_ERR_UNSUPPORTED, "Conv: bf16 storage needs the BF16 tensor-core path");
  const int bk = igemm_block_k(p->prec, a_bf16);
  p->a_bf16 = a_bf16;
  p->out_bf16 = out_bf16;
  p->dual = true;
  p->d2 = r2;
  p->cs2 = cs2;
  p->kb_split = (int)(a.c / bk);
  p->K = (int)(a.c + r2.c);
  p->kpad = p->K;
  p->num_kb = p->K / bk;
  choose_tiling(h, p, false);
  const size_t esz = p->prec == kPrecBF16 ? 2 : 4;
  const size_t wbytes = align_up((size_t)CO * p->kpad * esz);
  size_t need = wbytes * (p->prec == kPrec3xTF32 ? 2 : 1);
  const size_t off_s1 = need;
  need += align_up(CO * sizeof(float));
  const size_t off_s2 = need;
  need += align_up(CO * sizeof(float));
  const size_t off_t1 = need;
  need += align_up(CO * sizeof(float));
  const size_t off_t2 = need;
  need += align_up(CO * sizeof(float));
  p->weight_bytes = (int64_t)need;
  const size_t off_split = (!scratch && !scratch_used && p->split_bytes) ? need : 0;
  if (off_split) need += align_up(p->split_bytes);
  if (!scratch && scratch_used) {
    *scratch_used = need;
    return ONNXB200_OK;
  }
  uint8_t* basep = nullptr;
  if (scratch) {
    if (need > scratch_bytes)
      return set_error(h, ONNXB200_ERR_RESOURCE_EXHAUSTED, "Conv: scratch too small for packed weights");
    basep = static_cast<uint8_t*>(scratch);
    if (scratch_used) *scratch_used = need;
  } else {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&basep), need);
    if (e != cudaSuccess) return cuda_check(h, e, "conv plan allocation");
  }
  cudaStream_t st = h->stream;
  p->w_hi = basep;
  p->w_lo = p->prec == kPrec3xTF32 ? basep + wbytes : nullptr;
  p->w_oihw = nullptr;
  float* s1 = reinterpret_cast<float*>(basep + off_s1);
  float* s2 = reinterpret_cast<float*>(basep + off_s2);
  float* t1 = reinterpret_cast<float*>(basep + off_t1);
  float* t2 = reinterpret_cast<float*>(basep + off_t2);
  p->split_ws = off_split ? reinterpret_cast<float*>(basep + off_split) : nullptr;
  // each branch's BatchNormalization as scale / shift; the scales go into the
  // packed weights, the shifts are added: y = (s1 W1) x1 + (s2 W2) x2 + t1 + t2
  rc = bn_fold_launch(bn1.scale, bn1.bias, bn1.mean, bn1.var, bn1.conv_bias, bn1.eps, CO, s1, t1, st);
  if (!rc) rc = bn_fold_launch(bn2.scale, bn2.bias, bn2.mean, bn2.var, bn2.conv_bias, bn2.eps, CO, s2, t2, st);
  if (!rc) rc = pack_dual_b_launch(w1, s1, (int)a.c, w2, s2, (int)r2.c, CO, p->prec, p->w_hi, p->w_lo, st);
  if (!rc) rc = vec_add_launch(t1, t2, t1, CO, st);
  h->launches += 4;
  if (rc) return cuda_check(h, (cudaError_t)rc, "two-source weight packing");
  p->scale = nullptr;
  p->shift = t1;
  rc = encode_weight_map(h, &p->tm_hi, p->w_hi, CO, p->kpad, p->prec, p->bn, bk);
  if (rc) return rc;
  return encode_weight_map(h, &p->tm_lo, p->w_lo ? p->w_lo : p->w_hi, CO, p->kpad, p->prec, p->bn, bk);
}

bool dual_conv_supported(const onnxb200_conv_desc& a, int cs1, const onnxb200_conv_desc& b, int cs2) {
  auto one_by_one = [](const onnxb200_conv_desc& d) {
    return d.kh == 1 && d.kw == 1 && d.group == 1 && d.pad_top == 0 && d.pad_left == 0 && d.pad_bottom == 0 &&
           d.pad_right == 0 && d.dil_h == 1 && d.dil_w == 1 && d.auto_pad == ONNXB200_AUTOPAD_NOTSET;
  };
  return one_by_one(a) && one_by_one(b) && a.stride_h == 1 && a.stride_w == 1 && b.stride_h == b.stride_w &&
         b.stride_h <= 8 && a.c_out == b.c_out && a.n == b.n && cs1 == a.c && cs2 == b.c && a.c % 32 == 0 &&
         b.c % 32 == 0 && a.c_out % 4 == 0 && a.precision != kPrecFP32 && a.precision == b.precision;
}

int conv_dual_exec_nhwc(onnxb200_handle* h, const onnxb200_conv_plan* p, const float* x1, const float* x2,
                        float* y, float* split_ws) {
  const onnxb200_conv_desc& d = p->d;
  if (!p->dual) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: not a two-source plan");
  if (d.n == 0) return ONNXB200_OK;
  IgemmParams q{};
  q.x = x1;
  q.Hin = (int)d.h;
  q.Win = (int)d.w;
  q.Cs = p->cs_in;
  q.OH = (int)p->oh;
  q.OW = (int)p->ow;
  q.KW = 1;
  q.sh = q.sw = 1;
  q.dh = q.dw = 1;
  q.M = (int)(d.n * p->oh * p->ow);
  q.Nc = (int)d.c_out;
  q.K = p->K;
  q.num_kb = p->num_kb;
  q.batches = 1;
  q.y = y;
  q.ldy = (int)d.c_out;
  q.scale = p->scale;
  q.shift = p->shift;
  q.relu = (d.epilogue & ONNXB200_EPI_RELU) != 0;
  q.status = h->d_status;
  q.m_tiles = (q.M + 127) / 128;
  q.n_tiles = (q.Nc + p->bn - 1) / p->bn;
  q.a_mode = kALoadTma2d;
  q.a_bf16 = p->a_bf16;
  q.out_bf16 = p->out_bf16;
  q.kb_split = p->kb_split;
  q.x2 = x2;
  q.H2 = (int)p->d2.h;
  q.W2 = (int)p->d2.w;
  q.Cs2 = p->cs2;
  q.s2 = (int)p->d2.stride_h;
  IgemmParams v = second_source_view(q);
  q.a_mode2 = pick_a_mode(v, p->prec);
  v.a_mode = q.a_mode2;
  if (q.a_mode2 != kALoadTma2d && q.a_mode2 != kALoadIm2col)
    return set_error(h, ONNXB200_ERR_UNSUPPORTED, "Conv: second source cannot be read by TMA");
  CUtensorMap am{}, am2{};
  int er = encode_a_map(q, (int)d.n * q.Hin * q.Win, &am);
  if (!er) er = encode_a_map(v, q.a_mode2 == kALoadTma2d ? (int)d.n * q.H2 * q.W2 : (int)d.n, &am2);
  if (er) return set_error(h, ONNXB200_ERR_EXECUTION, "Conv: A tensor map encode failed: " + std::to_string(er));
  float* ws = split_ws ? split_ws : p->split_ws;
  const int rc = igemm_launch_split(q, ws ? p->ksplit : 1, p->split_mt, ws, p->tm_hi, p->tm_lo, am, am2,
                                    p->prec, p->bn, h->num_sms, h->stream);
  h->launches += (ws && p->ksplit > 1) ? (p->split_mt > 0 ? 3 : 2) : 1;
  if (rc) return cuda_check(h, (cudaError_t)rc, "Conv launch");
  return ONNXB200_OK;
}

int gemm_tc_run(onnxb200_handle* h, const GemmCall& c, const void* b_hi, const void* b_lo,
                int b_rows, int kpad, int prec) {
  IgemmParams q{};
  q.x = c.a;
  q.Hin = 1;
  q.Win = c.M;
  q.Cs = c.K;
  q.OH = 1;
  q.OW = c.M;
  q.KW = 1;
  q.sh = q.sw = 1;
  q.ph = q.pw = 0;
  q.dh = q.dw = 1;
  q.M = c.M;
  q.Nc = c.N;
  q.K = c.K;
  q.num_kb = kpad / igemm_block_k(prec);
  q.batches = c.batches;
  q.a_off = c.a_off;
  q.b_row = c.b_row;
  q.y_bstride = c.y_bstride;
  q.y = c.y;
  q.ldy = c.ldy;
  q.scale = c.scale;
  q.shift = c.shift;
  q.res = c.res;
  q.ldr = c.ldr;
  q.relu = c.relu;
  q.status = h->d_status;
  int bn = igemm_pick_bn(q, prec, h->num_sms), ks = 1, smt = 0;
  if (c.split_ws) {
    int b2 = bn, k2 = 1, m2 = 0;
    igemm_pick_split(q, q.res != nullptr, prec, h->num_sms, &b2, &k2, &m2);
    if (k2 > 1 && (size_t)k2 * (q.M - m2 * 128) * q.Nc * sizeof(float) <= c.split_bytes) {
      bn = b2;
      ks = k2;
      smt = m2;
    }
  }
  q.m_tiles = (q.M + 127) / 128;
  q.n_tiles = (q.Nc + bn - 1) / bn;
  CUtensorMap thi, tlo;
  int rc = encode_weight_map(h, &thi, b_hi, b_rows, kpad, prec, bn);
  if (rc) return rc;
  rc = encode_weight_map(h, &tlo, b_lo ? b_lo : b_hi, b_rows, kpad, prec, bn);
  if (rc) return rc;
  q.a_mode = pick_a_mode(q, prec);
  CUtensorMap am{};
  if (q.a_mode != kALoadGather) {
    const int er = encode_a_map(q, c.a_rows > 0 ? c.a_rows : c.M, &am);
    if (er) return set_error(h, ONNXB200_ERR_EXECUTION, "GEMM: A tensor map encode failed: " + std::to_string(er));
  }
  rc = igemm_launch_split(q, ks, smt, c.split_ws, thi, tlo, am, am, prec, bn, h->num_sms, h->stream);
  h->launches += ks > 1 ? (smt > 0 ? 3 : 2) : 1;
  if (rc) return cuda_check(h, (cudaError_t)rc, "GEMM launch");
  return ONNXB200_OK;
}

size_t gemm_split_bytes(const onnxb200_handle* h, int M, int N, int kpad, int prec, bool residual) {
  if (prec == kPrecFP32) return 0;
  IgemmParams q{};
  q.M = M;
  q.Nc = N;
  q.batches = 1;
  q.num_kb = kpad / igemm_block_k(prec);
  int bn = 128, ks = 1, smt = 0;
  igemm_pick_split(q, residual, prec, h->num_sms, &bn, &ks, &smt);
  return ks > 1 ? (size_t)ks * (M - smt * 128) * N * sizeof(float) : 0;
}

}  // namespace ob2

// =====================================================================================
// extern "C"
// =====================================================================================
extern "C" {

int onnxb200_version(void) { return 100; }

void onnxb200_default_options(onnxb200_options* o) {
  if (!o) return;
  o->precision = ONNXB200_PREC_3XTF32;
  o->workspace_bytes = 64ull << 20;
  o->use_cuda_graph = 1;
  o->wait_timeout_ms = 60000;
}

const char* onnxb200_status_string(int s) {
  switch (s) {
    case ONNXB200_OK: return "ok";
    case ONNXB200_ERR_VALIDATION: return "validation error";
    case ONNXB200_ERR_EXECUTION: return "execution error";
    case ONNXB200_ERR_UNSUPPORTED: return "unsupported feature";
    case ONNXB200_ERR_TIMEOUT: return "operation timed out";
    case ONNXB200_ERR_RESOURCE_EXHAUSTED: return "resource exhausted";
    case ONNXB200_ERR_INVALID_GRAPH: return "invalid graph structure";
    case ONNXB200_ERR_INVALID_OPERATOR: return "invalid operator";
    case ONNXB200_ERR_CANCELLED: return "execution cancelled";
    case ONNXB200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case ONNXB200_ERR_IO: return "I/O error";
    case ONNXB200_ERR_PROTOBUF: return "protobuf parsing error";
    case ONNXB200_ERR_INVALID_MODEL: return "invalid ONNX model";
    default: return "unknown status";
  }
}

int onnxb200_create(int device, const onnxb200_options* opts, onnxb200_handle** out) {
  if (!out) return ONNXB200_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  onnxb200_handle* h = new (std::nothrow) onnxb200_handle();
  if (!h) return ONNXB200_ERR_RESOURCE_EXHAUSTED;
  onnxb200_default_options(&h->opts);
  if (opts) {
    h->opts = *opts;
    if (h->opts.workspace_bytes == 0) h->opts.workspace_bytes = 64ull << 20;
    if (h->opts.wait_timeout_ms <= 0) h->opts.wait_timeout_ms = 60000;
    if (h->opts.precision < 0 || h->opts.precision > 3) h->opts.precision = ONNXB200_PREC_3XTF32;
  }
  h->device = device;
  const char* dbg = std::getenv("ONNXB200_DEBUG_SYNC");
  h->debug_sync = dbg && dbg[0] == '1';
  int rc = ONNXB200_OK;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0) {
      delete h;
      return ONNXB200_ERR_UNSUPPORTED;  // built for sm_100a only
    }
    cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
    // A blocking stream: work on it is ordered with the legacy default stream,
    // so callers that use the default stream (torch's default, plain
    // cudaMemcpy) see results in order without extra synchronisation.
    e = cudaStreamCreateWithFlags(&h->own_stream, cudaStreamDefault);
  }
  if (e == cudaSuccess) {
    h->stream = h->own_stream;
    e = cudaMalloc(&h->d_status, 256);
  }
  if (e == cudaSuccess) e = cudaMemsetAsync(h->d_status, 0, 256, h->stream);
  if (e == cudaSuccess) e = cudaMalloc(&h->ws, h->opts.workspace_bytes);
  if (e == cudaSuccess) {
    h->ws_bytes = h->opts.workspace_bytes;
    e = cudaStreamSynchronize(h->stream);
  }
  if (e != cudaSuccess) {
    rc = e == cudaErrorMemoryAllocation ? ONNXB200_ERR_RESOURCE_EXHAUSTED : ONNXB200_ERR_EXECUTION;
    if (h->ws) cudaFree(h->ws);
    if (h->d_status) cudaFree(h->d_status);
    if (h->own_stream) cudaStreamDestroy(h->own_stream);
    delete h;
    return rc;
  }
  *out = h;
  return ONNXB200_OK;
}

int onnxb200_destroy(onnxb200_handle* h) {
  if (!h) return ONNXB200_ERR_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  if (h->ws) cudaFree(h->ws);
  if (h->d_status) cudaFree(h->d_status);
  if (h->own_stream) cudaStreamDestroy(h->own_stream);
  delete h;
  return ONNXB200_OK;
}

const char* onnxb200_last_error(const onnxb200_handle* h) {
  return h ? h->last_error.c_str() : "null handle";
}

int onnxb200_set_stream(onnxb200_handle* h, void* s) {
  if (!h) return ONNXB200_ERR_INVALID_ARGUMENT;
  h->stream = s ? static_cast<cudaStream_t>(s) : h->own_stream;
  return ONNXB200_OK;
}

void* onnxb200_get_stream(onnxb200_handle* h) { return h ? (void*)h->stream : nullptr; }

int64_t onnxb200_kernel_launches(const onnxb200_handle* h) { return h ? h->launches : -1; }

int onnxb200_malloc(onnxb200_handle* h, size_t bytes, void** ptr) {
  if (!h || !ptr) return ONNXB200_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  cudaSetDevice(h->device);
  if (bytes == 0) return ONNXB200_OK;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) {
    *ptr = nullptr;
    return cuda_check(h, e, "device allocation");
  }
  return ONNXB200_OK;
}

int onnxb200_free(onnxb200_handle* h, void* ptr) {
  if (!h) return ONNXB200_ERR_INVALID_ARGUMENT;
  if (!ptr) return ONNXB200_OK;
  cudaSetDevice(h->device);
  return cuda_check(h, cudaFree(ptr), "device free");
}

int onnxb200_memcpy(onnxb200_handle* h, void* dst, const void* src, size_t bytes, int kind) {
  if (!h || (bytes && (!dst || !src)) || kind < 0 || kind > 2) return ONNXB200_ERR_INVALID_ARGUMENT;
  if (bytes == 0) return ONNXB200_OK;
  cudaSetDevice(h->device);
  const cudaMemcpyKind k = kind == ONNXB200_COPY_H2D   ? cudaMemcpyHostToDevice
                           : kind == ONNXB200_COPY_D2H ? cudaMemcpyDeviceToHost
                                                       : cudaMemcpyDeviceToDevice;
  return cuda_check(h, cudaMemcpyAsync(dst, src, bytes, k, h->stream), "copy");
}

int onnxb200_num_sms(const onnxb200_handle* h) { return h ? h->num_sms : -1; }

int onnxb200_synchronize(onnxb200_handle* h) {
  if (!h) return ONNXB200_ERR_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  // Bounded wait: poll the stream instead of blocking forever.
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaStreamQuery(h->stream);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return cuda_check(h, q, "stream");
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (ms > h->opts.wait_timeout_ms)
      return set_error(h, ONNXB200_ERR_TIMEOUT, "synchronize: stream did not finish in time");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  int status = 0;
  cudaError_t e = cudaMemcpy(&status, h->d_status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_check(h, e, "status read");
  if (status != 0) {
    cudaMemset(h->d_status, 0, sizeof(int));
    return set_error(h, status, std::string("device reported: ") + onnxb200_status_string(status));
  }
  return ONNXB200_OK;
}

// ---------------------------------------------------------------------------------- Conv
int onnxb200_conv2d_output_shape(const onnxb200_conv_desc* d, int64_t out[4]) {
  onnxb200_conv_desc r;
  int64_t oh, ow;
  onnxb200_handle tmp;
  int rc = resolve_conv_desc(&tmp, d, &r, &oh, &ow);
  if (rc) return rc;
  out[0] = r.n;
  out[1] = r.c_out;
  out[2] = oh;
  out[3] = ow;
  return ONNXB200_OK;
}

int onnxb200_conv_plan_create(onnxb200_handle* h, const onnxb200_conv_desc* d, const float* w,
                              const float* bias, const float* bn_scale, const float* bn_bias,
                              const float* bn_mean, const float* bn_var, onnxb200_conv_plan** out) {
  if (!h || !out) return ONNXB200_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  cudaSetDevice(h->device);
  onnxb200_conv_plan* p = new (std::nothrow) onnxb200_conv_plan();
  if (!p) return ONNXB200_ERR_RESOURCE_EXHAUSTED;
  // NHWC plans read the caller's NHWC input directly (channel stride c);
  // NCHW plans repack into a channel-padded NHWC copy first.
  const int layout = d ? d->layout : 0;
  const int cs = layout == ONNXB200_LAYOUT_NHWC ? (int)d->c : (int)((d->c + 3) / 4 * 4);
  int rc = conv_plan_init(h, d, cs, w, bias, bn_scale, bn_bias, bn_mean, bn_var, p, nullptr, 0,
                          nullptr);
  if (rc) {
    delete p;
    return rc;
  }
  *out = p;
  return ONNXB200_OK;
}

int onnxb200_conv_plan_destroy(onnxb200_conv_plan* p) {
  if (!p) return ONNXB200_ERR_INVALID_ARGUMENT;
  void* base = p->use_tc ? p->w_hi : (void*)p->w_oihw;
  if (base) cudaFree(base);
  delete p;
  return ONNXB200_OK;
}

// Runs a plan on tensors of the plan's layout, repacking NCHW through the workspace.
static int conv_run_layout(onnxb200_handle* h, const onnxb200_conv_plan* p, const float* x,
                           const float* residual, float* y, size_t ws_offset) {
  const onnxb200_conv_desc& d = p->d;
  if (d.layout == ONNXB200_LAYOUT_NHWC) return conv_plan_exec_nhwc(h, p, x, residual, y);
  const size_t xb = align_up((size_t)d.n * d.h * d.w * p->cs_in * sizeof(float));
  const size_t yb = align_up((size_t)d.n * p->oh * p->ow * d.c_out * sizeof(float));
  const bool has_res = (d.epilogue & ONNXB200_EPI_RESIDUAL) && residual;
  int rc = ensure_workspace(h, ws_offset + xb + yb * (has_res ? 2 : 1));
  if (rc) return rc;
  uint8_t* ws = static_cast<uint8_t*>(h->ws) + ws_offset;
  float* xn = reinterpret_cast<float*>(ws);
  float* yn = reinterpret_cast<float*>(ws + xb);
  float* rn = has_res ? reinterpret_cast<float*>(ws + xb + yb) : nullptr;
  rc = nchw_to_nhwc_launch(x, (int)d.n, (int)d.c, (int)d.h, (int)d.w, p->cs_in, xn, h->stream);
  h->launches++;
  if (rc) return cuda_check(h, (cudaError_t)rc, "NCHW->NHWC");
  if (rn) {
    rc = nchw_to_nhwc_launch(residual, (int)d.n, (int)d.c_out, (int)p->oh, (int)p->ow, (int)d.c_out,
                             rn, h->stream);
    h->launches++;
    if (rc) return cuda_check(h, (cudaError_t)rc, "NCHW->NHWC");
  }
  rc = conv_plan_exec_nhwc(h, p, xn, rn, yn);
  if (rc) return rc;
  rc = nhwc_to_nchw_launch(yn, (int)d.n, (int)d.c_out, (int)p->oh, (int)p->ow, (int)d.c_out, y,
                           h->stream);
  h->launches++;
  if (rc) return cuda_check(h, (cudaError_t)rc, "NHWC->NCHW");
  return ONNXB200_OK;
}

int onnxb200_conv_plan_run(onnxb200_handle* h, const onnxb200_conv_plan* p, const float* x,
                           const float* residual, float* y) {
  if (!h || !p || !x || !y) return ONNXB200_ERR_INVALID_ARGUMENT;
  return conv_run_layout(h, p, x, residual, y, 0);
}

// ---------------------------------------------------------------- 1-D / 2-D / 3-D
namespace {
// Resolved geometry of an N-d convolution (spatial dims padded to 3 with ones
// in front: 1-D is [1, 1, L], 2-D is [1, H, W]).
struct ConvNd {
  int sp;
  int64_t n, c, co, g;
  int64_t in[3], k[3], s[3], pb[3], pe[3], dl[3], out[3];
};

int resolve_conv_nd(onnxb200_handle* h, const onnxb200_conv_nd_desc* d, ConvNd* r) {
  if (!d) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "null conv descriptor");
  // compute_conv (src/ops/nn/conv.rs:546-565): rank 3 to 5 (1 to 3 spatial dims)
  if (d->spatial < 1 || d->spatial > 3)
    return set_error(h, ONNXB200_ERR_VALIDATION, "Conv supports only 1D, 2D, and 3D convolutions");
  r->sp = d->spatial;
  r->n = d->n;
  r->c = d->c;
  r->co = d->c_out;
  r->g = d->group > 0 ? d->group : 1;
  if (r->n < 0 || r->c <= 0 || r->co <= 0) return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: non-positive dimension");
  if (r->c % r->g != 0 || r->co % r->g != 0)
    return set_error(h, ONNXB200_ERR_VALIDATION, "Input and output channels must be divisible by groups");
  const int off = 3 - r->sp;
  for (int i = 0; i < 3; ++i) {
    const int j = i - off;  // index into the descriptor's arrays
    const bool used = j >= 0;
    r->in[i] = used ? d->in[j] : 1;
    r->k[i] = used ? d->kernel[j] : 1;
    r->s[i] = used && d->stride[j] > 0 ? d->stride[j] : 1;
    r->dl[i] = used && d->dilation[j] > 0 ? d->dilation[j] : 1;
    r->pb[i] = used ? d->pad_begin[j] : 0;
    r->pe[i] = used ? d->pad_end[j] : 0;
    if (r->in[i] <= 0 || r->k[i] <= 0) return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: non-positive dimension");
    if (used && (d->auto_pad == ONNXB200_AUTOPAD_SAME_UPPER || d->auto_pad == ONNXB200_AUTOPAD_SAME_LOWER)) {
      // calculate_same_padding (src/ops/nn/conv.rs:426-458)
      const int64_t dk = (r->k[i] - 1) * r->dl[i] + 1;
      const int64_t o = (r->in[i] + r->s[i] - 1) / r->s[i];
      const int64_t need = (o - 1) * r->s[i] + dk - r->in[i];
      const int64_t half = need > 0 ? need / 2 : 0, rest = need > 0 ? need - half : 0;
      r->pb[i] = d->auto_pad == ONNXB200_AUTOPAD_SAME_UPPER ? half : rest;
      r->pe[i] = d->auto_pad == ONNXB200_AUTOPAD_SAME_UPPER ? rest : half;
    } else if (d->auto_pad == ONNXB200_AUTOPAD_VALID) {
      r->pb[i] = r->pe[i] = 0;
    } else if (d->auto_pad != ONNXB200_AUTOPAD_NOTSET && d->auto_pad != ONNXB200_AUTOPAD_SAME_UPPER &&
               d->auto_pad != ONNXB200_AUTOPAD_SAME_LOWER) {
      return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: unknown auto_pad");
    }
    if (r->pb[i] < 0 || r->pe[i] < 0) return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: negative padding");
    r->out[i] = conv_out_dim(r->in[i], r->k[i], r->s[i], r->pb[i], r->pe[i], r->dl[i]);
    if (r->out[i] <= 0) return set_error(h, ONNXB200_ERR_VALIDATION, "Conv: kernel larger than padded input");
  }
  int64_t in_el = r->n * r->c, out_el = r->n * r->co;
  for (int i = 0; i < 3; ++i) {
    in_el *= r->in[i];
    out_el *= r->out[i];
  }
  if (in_el > (int64_t)INT32_MAX * 4 || out_el > (int64_t)INT32_MAX * 4 ||
      r->co * (r->c / r->g) * r->k[0] * r->k[1] * r->k[2] > (int64_t)INT32_MAX)
    return set_error(h, ONNXB200_ERR_UNSUPPORTED, "Conv: tensor too large");
  return ONNXB200_OK;
}
}  // namespace

int onnxb200_conv_nd_output_shape(const onnxb200_conv_nd_desc* d, int64_t out[5], int* rank) {
  if (!d || !out || !rank) return ONNXB200_ERR_INVALID_ARGUMENT;
  onnxb200_handle tmp;
  ConvNd r;
  int rc = resolve_conv_nd(&tmp, d, &r);
  if (rc) return rc;
  *rank = r.sp + 2;
  out[0] = r.n;
  out[1] = r.co;
  for (int i = 0; i < r.sp; ++i) out[2 + i] = r.out[3 - r.sp + i];
  return ONNXB200_OK;
}

int onnxb200_conv_nd(onnxb200_handle* h, const onnxb200_conv_nd_desc* d, const float* x, const float* w,
                     const float* bias, float* y) {
  if (!h || !d) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null argument");
  cudaSetDevice(h->device);
  ConvNd r;
  int rc = resolve_conv_nd(h, d, &r);
  if (rc) return rc;
  if (r.n == 0) return ONNXB200_OK;
  if (!x || !w || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null argument");
  if (r.sp <= 2) {
    // 1-D (NCL) is the 2-D convolution of an [N, C, 1, L] tensor with [CO, C/g, 1, k]
    // filters: the same memory, run on the tensor-core path
    onnxb200_conv_desc c{};
    c.n = r.n;
    c.c = r.c;
    c.h = r.in[1];
    c.w = r.in[2];
    c.c_out = r.co;
    c.kh = r.k[1];
    c.kw = r.k[2];
    c.stride_h = r.s[1];
    c.stride_w = r.s[2];
    c.pad_top = r.pb[1];
    c.pad_left = r.pb[2];
    c.pad_bottom = r.pe[1];
    c.pad_right = r.pe[2];
    c.dil_h = r.dl[1];
    c.dil_w = r.dl[2];
    c.group = r.g;
    c.auto_pad = ONNXB200_AUTOPAD_NOTSET;
    c.layout = ONNXB200_LAYOUT_NCHW;
    c.epilogue = (bias ? ONNXB200_EPI_BIAS : 0) | (d->relu ? ONNXB200_EPI_RELU : 0);
    c.precision = ONNXB200_PREC_DEFAULT;
    return onnxb200_conv2d(h, &c, x, w, bias, nullptr, nullptr, nullptr, nullptr, nullptr, y);
  }
  Conv3dArgs a{};
  a.N = (int)r.n;
  a.C = (int)r.c;
  a.CO = (int)r.co;
  a.G = (int)r.g;
  a.D = (int)r.in[0];
  a.H = (int)r.in[1];
  a.W = (int)r.in[2];
  a.KD = (int)r.k[0];
  a.KH = (int)r.k[1];
  a.KW = (int)r.k[2];
  a.OD = (int)r.out[0];
  a.OH = (int)r.out[1];
  a.OW = (int)r.out[2];
  a.sd = (int)r.s[0];
  a.sh = (int)r.s[1];
  a.sw = (int)r.s[2];
  a.pd = (int)r.pb[0];
  a.ph = (int)r.pb[1];
  a.pw = (int)r.pb[2];
  a.dd = (int)r.dl[0];
  a.dh = (int)r.dl[1];
  a.dw = (int)r.dl[2];
  a.relu = d->relu ? 1 : 0;
  rc = conv3d_direct_launch(x, w, bias, y, a, h->stream);
  h->launches++;
  if (rc) return cuda_check(h, (cudaError_t)rc, "Conv3d launch");
  return ONNXB200_OK;
}

int onnxb200_conv2d(onnxb200_handle* h, const onnxb200_conv_desc* d, const float* x,
                    const float* w, const float* bias, const float* bn_scale, const float* bn_bias,
                    const float* bn_mean, const float* bn_var, const float* residual, float* y) {
  if (!h || !d) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null argument");
  cudaSetDevice(h->device);
  const int cs = d->layout == ONNXB200_LAYOUT_NHWC ? (int)d->c : (int)((d->c + 3) / 4 * 4);
  // Packed weights go to the front of the workspace; activation repacks follow.
  onnxb200_conv_desc r;
  int64_t oh, ow;
  int rc = resolve_conv_desc(h, d, &r, &oh, &ow);
  if (rc) return rc;
  if (r.n == 0) return ONNXB200_OK;  // empty batch: nothing to compute (buffers may be null)
  if (!x || !w || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Conv: null argument");
  const size_t wneed = align_up((size_t)r.c_out * ((r.kh * r.kw * cs + 31) / 32 * 32) * 4) * 2 +
                       align_up((size_t)r.c_out * (r.c / r.group) * r.kh * r.kw * 4) +
                       2 * align_up(r.c_out * 4) + kAlign;
  // Reserve the activation repacks too, so the workspace is not regrown (and
  // the packed weights freed) between packing and running.
  size_t aneed = 0;
  if (r.layout == ONNXB200_LAYOUT_NCHW) {
    const size_t yb = align_up((size_t)r.n * oh * ow * r.c_out * sizeof(float));
    aneed = align_up((size_t)r.n * r.h * r.w * cs * sizeof(float)) +
            yb * (((r.epilogue & ONNXB200_EPI_RESIDUAL) && residual) ? 2 : 1);
  }
  rc = ensure_workspace(h, wneed + aneed);
  if (rc) return rc;
  onnxb200_conv_plan p;
  size_t used = 0;
  rc = conv_plan_init(h, d, cs, w, bias, bn_scale, bn_bias, bn_mean, bn_var, &p, h->ws, h->ws_bytes,
                      &used);
  if (rc) return rc;
  return conv_run_layout(h, &p, x, residual, y, align_up(used));
}

// ---------------------------------------------------------------------------------- MatMul
int onnxb200_matmul_output_shape(const int64_t* as, int ra, const int64_t* bs, int rb,
                                 int64_t* out, int* ro) {
  // validate_matmul_shapes (src/ops/math/matmul.rs:401-487)
  if (!as || !bs || !out || !ro) return ONNXB200_ERR_INVALID_ARGUMENT;
  if (ra <= 0 || rb <= 0 || ra > 8 || rb > 8) return ONNXB200_ERR_VALIDATION;
  if (ra == 1 && rb == 1) {
    if (as[0] != bs[0]) return ONNXB200_ERR_VALIDATION;
    *ro = 0;
    return ONNXB200_OK;
  }
  if (ra == 1) {
    if (as[0] != bs[rb - 2]) return ONNXB200_ERR_VALIDATION;
    for (int i = 0; i < rb - 2; ++i) out[i] = bs[i];
    out[rb - 2] = bs[rb - 1];
    *ro = rb - 1;
    return ONNXB200_OK;
  }
  if (rb == 1) {
    if (as[ra - 1] != bs[0]) return ONNXB200_ERR_VALIDATION;
    for (int i = 0; i < ra - 2; ++i) out[i] = as[i];
    out[ra - 2] = as[ra - 2];
    *ro = ra - 1;
    return ONNXB200_OK;
  }
  if (as[ra - 1] != bs[rb - 2]) return ONNXB200_ERR_VALIDATION;
  const int na = ra - 2, nb = rb - 2, r = std::max(na, nb);
  for (int i = 0; i < r; ++i) {
    // broadcast_batch_dims (src/ops/math/matmul.rs:497-546)
    const int64_t da = i >= r - na ? as[i - (r - na)] : 1;
    const int64_t db = i >= r - nb ? bs[i - (r - nb)] : 1;
    if (da == 1)
      out[i] = db;
    else if (db == 1 || da == db)
      out[i] = da;
    else
      return ONNXB200_ERR_VALIDATION;
  }
  out[r] = as[ra - 2];
  out[r + 1] = bs[rb - 1];
  *ro = r + 2;
  return ONNXB200_OK;
}

// create_broadcast_indices (src/ops/math/matmul.rs:587-643) for one output batch.
static int64_t bcast_index(int64_t o, const int64_t* outd, int ro, const int64_t* in, int ri) {
  int64_t idx = 0, stride = 1, rem = o;
  for (int i = ro - 1; i >= 0; --i) {
    const int64_t d = outd[i];
    if (d == 0) continue;
    const int64_t coord = rem % d;
    rem /= d;
    const int j = i - (ro - ri);
    if (j >= 0) {
      if (in[j] != 1) idx += coord * stride;
      stride *= in[j];
    }
  }
  return idx;
}

int onnxb200_matmul(onnxb200_handle* h, const float* a, const int64_t* as, int ra, const float* b,
                    const int64_t* bs, int rb, const float* bias, int flags, int precision,
                    float* y) {
  if (!h || !a || !b || !y || !as || !bs)
    return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "MatMul: null argument");
  cudaSetDevice(h->device);
  int64_t outs[10];
  int ro = 0;
  if (onnxb200_matmul_output_shape(as, ra, bs, rb, outs, &ro) != ONNXB200_OK)
    return set_error(h, ONNXB200_ERR_VALIDATION, "MatMul: incompatible shapes");
  // Promote 1-D operands (compute_vector_matmul, src/ops/math/matmul.rs:282-398).
  std::vector<int64_t> A(as, as + ra), B(bs, bs + rb);
  if (ra == 1) A = {1, as[0]};
  if (rb == 1) B = {bs[0], 1};
  const int64_t M = A[A.size() - 2], K = A[A.size() - 1], N = B[B.size() - 1];
  std::vector<int64_t> ab(A.begin(), A.end() - 2), bb(B.begin(), B.end() - 2);
  const int r = (int)std::max(ab.size(), bb.size());
  std::vector<int64_t> ob(r);
  for (int i = 0; i < r; ++i) {
    const int64_t da = i >= r - (int)ab.size() ? ab[i - (r - ab.size())] : 1;
    const int64_t db = i >= r - (int)bb.size() ? bb[i - (r - bb.size())] : 1;
    ob[i] = da == 1 ? db : da;
  }
  int64_t nbatch = 1, nb_b = 1;
  for (auto v : ob) nbatch *= v;
  for (auto v : bb) nb_b *= v;
  if (nbatch == 0 || M == 0 || N == 0) return ONNXB200_OK;
  const int prec = resolve_prec(h, precision);
  std::vector<long long> aoff(nbatch), boff(nbatch);
  std::vector<int> brow(nbatch);
  for (int64_t i = 0; i < nbatch; ++i) {
    const int64_t ia = bcast_index(i, ob.data(), r, ab.data(), (int)ab.size());
    const int64_t ib = bcast_index(i, ob.data(), r, bb.data(), (int)bb.size());
    aoff[i] = ia * M * K;
    boff[i] = ib * K * N;
    brow[i] = (int)(ib * N);
  }
  const bool relu = (flags & ONNXB200_EPI_RELU) != 0;
  const bool tc = prec != kPrecFP32 && K % 4 == 0 && N % 4 == 0 && K > 0 &&
                  (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(y) & 15) == 0 && (!bias || (reinterpret_cast<uintptr_t>(bias) & 15) == 0) &&
                  M * K * nbatch < (1ll << 40) && nb_b * N < (1ll << 31);
  const size_t offs_bytes = align_up(nbatch * sizeof(long long)) * 2 + align_up(nbatch * sizeof(int));
  if (!tc) {
    int rc = ensure_workspace(h, offs_bytes);
    if (rc) return rc;
    uint8_t* ws = static_cast<uint8_t*>(h->ws);
    long long* d_aoff = reinterpret_cast<long long*>(ws);
    long long* d_boff = reinterpret_cast<long long*>(ws + align_up(nbatch * sizeof(long long)));
    cudaMemcpyAsync(d_aoff, aoff.data(), nbatch * sizeof(long long), cudaMemcpyHostToDevice, h->stream);
    cudaMemcpyAsync(d_boff, boff.data(), nbatch * sizeof(long long), cudaMemcpyHostToDevice, h->stream);
    rc = gemm_simt_launch(a, b, (int)nbatch, d_aoff, d_boff, M * N, (int)M, (int)N, (int)K, (int)K,
                          (int)N, 0, 0, nullptr, bias, nullptr, 0, relu, y, (int)N, h->stream);
    h->launches++;
    if (rc) return cuda_check(h, (cudaError_t)rc, "MatMul (CUDA cores)");
    return ONNXB200_OK;
  }
  const int kpad = igemm_kpad(K, prec);
  const size_t esz = prec == kPrecBF16 ? 2 : 4;
  const size_t wb = align_up((size_t)nb_b * N * kpad * esz);
  const size_t need = wb * (prec == kPrec3xTF32 ? 2 : 1) + offs_bytes;
  int rc = ensure_workspace(h, need);
  if (rc) return rc;
  uint8_t* ws = static_cast<uint8_t*>(h->ws);
  void* bhi = ws;
  void* blo = prec == kPrec3xTF32 ? ws + wb : nullptr;
  uint8_t* tail = ws + wb * (prec == kPrec3xTF32 ? 2 : 1);
  long long* d_aoff = reinterpret_cast<long long*>(tail);
  int* d_brow = reinterpret_cast<int*>(tail + 2 * align_up(nbatch * sizeof(long long)));
  // B[bb][k][n] -> packed row (bb*N + n), column k.
  rc = pack_b_launch(b, (int)(nb_b * N), (int)K, kpad, (int)K, (int)K, (int)N, K * N, 1, 0, N, prec,
                     bhi, blo, h->stream);
  h->launches++;
  if (rc) return cuda_check(h, (cudaError_t)rc, "MatMul pack");
  cudaMemcpyAsync(d_aoff, aoff.data(), nbatch * sizeof(long long), cudaMemcpyHostToDevice, h->stream);
  cudaMemcpyAsync(d_brow, brow.data(), nbatch * sizeof(int), cudaMemcpyHostToDevice, h->stream);
  GemmCall c;
  c.a = a;
  c.M = (int)M;
  c.N = (int)N;
  c.K = (int)K;
  c.batches = (int)nbatch;
  c.a_off = d_aoff;
  {
    int64_t arows = M;
    for (auto v : ab) arows *= v;
    c.a_rows = (int)arows;
  }
  c.b_row = d_brow;
  c.y_bstride = M * N;
  c.y = y;
  c.ldy = (int)N;
  c.shift = bias;
  c.relu = relu;
  return gemm_tc_run(h, c, bhi, blo, (int)(nb_b * N), kpad, prec);
}

// ---------------------------------------------------------------------------------- Gemm
__global__ void gemm_c_kernel(const float* c, long long cm, long long cn, float beta, int M, int N,
                              float* out) {
  const long long total = (long long)M * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / N, col = i % N;
    out[i] = beta * c[(cm == 1 ? 0 : r) * cn + (cn == 1 ? 0 : col)];
  }
}

__global__ void fill_kernel(float* p, float v, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

int onnxb200_gemm(onnxb200_handle* h, const float* a, const float* b, const float* c,
                  const int64_t* cs, int c_rank, int64_t m, int64_t n, int64_t k, int trans_a,
                  int trans_b, float alpha, float beta, int flags, int precision, float* y) {
  if (!h || !a || !b || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Gemm: null argument");
  cudaSetDevice(h->device);
  if (m < 0 || n < 0 || k < 0) return set_error(h, ONNXB200_ERR_VALIDATION, "Gemm: negative dimension");
  int64_t cm = 1, cn = 1;
  if (c) {
    if (c_rank == 1) {
      cn = cs[0];
    } else if (c_rank == 2) {
      cm = cs[0];
      cn = cs[1];
    } else if (c_rank != 0)
      return set_error(h, ONNXB200_ERR_VALIDATION, "Gemm: C must have rank <= 2");
    if ((cm != 1 && cm != m) || (cn != 1 && cn != n))
      return set_error(h, ONNXB200_ERR_VALIDATION, "Gemm: C is not broadcastable to [M, N]");
  }
  if (m == 0 || n == 0) return ONNXB200_OK;
  const int prec = resolve_prec(h, precision);
  const bool relu = (flags & ONNXB200_EPI_RELU) != 0;
  const bool use_c = c && beta != 0.f;
  const bool c_is_row = use_c && cm == 1;  // per-column (or scalar) addend
  const bool tc = prec != kPrecFP32 && k % 4 == 0 && n % 4 == 0 && k > 0 &&
                  (reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  const int kpad = igemm_kpad(k, prec);
  const size_t esz = prec == kPrecBF16 ? 2 : 4;
  const size_t wb = tc ? align_up((size_t)n * kpad * esz) : 0;
  const size_t ab = (tc && trans_a) ? align_up((size_t)m * k * 4) : 0;
  const size_t vb = align_up((size_t)n * 4);
  const size_t cb = (use_c && !c_is_row) ? align_up((size_t)m * n * 4) : 0;
  int rc = ensure_workspace(h, wb * 2 + ab + 2 * vb + cb);
  if (rc) return rc;
  uint8_t* ws = static_cast<uint8_t*>(h->ws);
  void* bhi = ws;
  void* blo = prec == kPrec3xTF32 ? ws + wb : nullptr;
  float* at = reinterpret_cast<float*>(ws + 2 * wb);
  float* scale = reinterpret_cast<float*>(ws + 2 * wb + ab);
  float* shift = reinterpret_cast<float*>(ws + 2 * wb + ab + vb);
  float* cfull = reinterpret_cast<float*>(ws + 2 * wb + ab + 2 * vb);
  cudaStream_t st = h->stream;
  const float* scale_p = nullptr;
  if (alpha != 1.f) {
    fill_kernel<<<(int)((n + 255) / 256), 256, 0, st>>>(scale, alpha, (int)n);
    h->launches++;
    scale_p = scale;
  }
  const float* shift_p = nullptr;
  const float* res_p = nullptr;
  if (use_c && c_is_row) {
    gemm_c_kernel<<<(int)((n + 255) / 256), 256, 0, st>>>(c, 1, cn, beta, 1, (int)n, shift);
    h->launches++;
    shift_p = shift;
  } else if (use_c) {
    gemm_c_kernel<<<(int)std::min<int64_t>((m * n + 255) / 256, 1 << 20), 256, 0, st>>>(c, cm, cn, beta, (int)m, (int)n, cfull);
    h->launches++;
    res_p = cfull;
  }
  if (!tc) {
    rc = gemm_simt_launch(a, b, 1, nullptr, nullptr, 0, (int)m, (int)n, (int)k,
                          trans_a ? (int)m : (int)k, trans_b ? (int)k : (int)n, trans_a, trans_b,
                          scale_p, shift_p, res_p, (int)n, relu, y, (int)n, st);
    h->launches++;
    if (rc) return cuda_check(h, (cudaError_t)rc, "Gemm (CUDA cores)");
    return ONNXB200_OK;
  }
  const float* arow = a;
  if (trans_a) {  // A is [K, M]: transpose to row-major [M, K]
    rc = nchw_to_nhwc_launch(a, 1, (int)k, 1, (int)m, (int)k, at, st);
    h->launches++;
    if (rc) return cuda_check(h, (cudaError_t)rc, "Gemm transpose");
    arow = at;
  }
  // B element (row n, col k): transB ? B[n][k] : B[k][n]
  rc = pack_b_launch(b, (int)n, (int)k, kpad, (int)k, (int)k, (int)n, 0, trans_b ? k : 1, 0,
                     trans_b ? 1 : n, prec, bhi, blo, st);
  h->launches++;
  if (rc) return cuda_check(h, (cudaError_t)rc, "Gemm pack");
  GemmCall g;
  g.a = arow;
  g.M = (int)m;
  g.N = (int)n;
  g.K = (int)k;
  g.batches = 1;
  g.y = y;
  g.ldy = (int)n;
  g.scale = scale_p;
  g.shift = shift_p;
  g.res = res_p;
  g.ldr = (int)n;
  g.relu = relu;
  return gemm_tc_run(h, g, bhi, blo, (int)n, kpad, prec);
}

// ---------------------------------------------------------------------------------- pooling
int onnxb200_maxpool2d(onnxb200_handle* h, int layout, int64_t n, int64_t c, int64_t hh,
                       int64_t ww, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t pt,
                       int64_t pl, int64_t pb, int64_t pr, int ceil_mode, const float* x, float* y,
                       int64_t* indices, int64_t out[4]) {
  if (!h || !x || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "MaxPool: null argument");
  cudaSetDevice(h->device);
  if (kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || pt < 0 || pl < 0 || pb < 0 || pr < 0)
    return set_error(h, ONNXB200_ERR_VALIDATION, "MaxPool: invalid attributes");
  // output size: pool.rs:343-344 (floor) / planner.rs:1230 (ceil_mode)
  int64_t oh, ow;
  if (ceil_mode) {
    oh = (hh + pt + pb - kh + sh - 1) / sh + 1;
    ow = (ww + pl + pr - kw + sw - 1) / sw + 1;
  } else {
    oh = (hh + pt + pb - kh) / sh + 1;
    ow = (ww + pl + pr - kw) / sw + 1;
  }
  if (hh + pt + pb < kh || ww + pl + pr < kw || oh <= 0 || ow <= 0)
    return set_error(h, ONNXB200_ERR_VALIDATION, "MaxPool: window larger than padded input");
  if (out) {
    out[0] = n;
    out[1] = c;
    out[2] = oh;
    out[3] = ow;
  }
  if (n == 0 || c == 0) return ONNXB200_OK;
  int rc;
  if (layout == ONNXB200_LAYOUT_NHWC) {
    rc = maxpool_nhwc_launch(x, (int)n, (int)c, (int)c, (int)hh, (int)ww, (int)kh, (int)kw, (int)sh,
                             (int)sw, (int)pt, (int)pl, (int)oh, (int)ow, y,
                             reinterpret_cast<long long*>(indices), h->stream);
    h->launches++;
    return rc ? cuda_check(h, (cudaError_t)rc, "MaxPool") : ONNXB200_OK;
  }
  const size_t xb = align_up((size_t)n * c * hh * ww * 4), yb = align_up((size_t)n * c * oh * ow * 4);
  rc = ensure_workspace(h, xb + yb);
  if (rc) return rc;
  float* xn = static_cast<float*>(h->ws);
  float* yn = reinterpret_cast<float*>(static_cast<uint8_t*>(h->ws) + xb);
  rc = nchw_to_nhwc_launch(x, (int)n, (int)c, (int)hh, (int)ww, (int)c, xn, h->stream);
  h->launches++;
  if (!rc) {
    rc = maxpool_nhwc_launch(xn, (int)n, (int)c, (int)c, (int)hh, (int)ww, (int)kh, (int)kw,
                             (int)sh, (int)sw, (int)pt, (int)pl, (int)oh, (int)ow, yn,
                             reinterpret_cast<long long*>(indices), h->stream);
    h->launches++;
  }
  if (!rc) {
    rc = nhwc_to_nchw_launch(yn, (int)n, (int)c, (int)oh, (int)ow, (int)c, y, h->stream);
    h->launches++;
  }
  return rc ? cuda_check(h, (cudaError_t)rc, "MaxPool") : ONNXB200_OK;
}

int onnxb200_global_avgpool(onnxb200_handle* h, int layout, int64_t n, int64_t c, int64_t hh,
                            int64_t ww, const float* x, float* y) {
  if (!h || !x || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "GlobalAveragePool: null argument");
  cudaSetDevice(h->device);
  if (n < 0 || c < 0 || hh <= 0 || ww <= 0)
    return set_error(h, ONNXB200_ERR_VALIDATION, "GlobalAveragePool: invalid shape");
  if (n == 0 || c == 0) return ONNXB200_OK;
  int rc;
  const float* xn = x;
  if (layout != ONNXB200_LAYOUT_NHWC && hh * ww > 1) {
    rc = ensure_workspace(h, align_up((size_t)n * c * hh * ww * 4));
    if (rc) return rc;
    float* t = static_cast<float*>(h->ws);
    rc = nchw_to_nhwc_launch(x, (int)n, (int)c, (int)hh, (int)ww, (int)c, t, h->stream);
    h->launches++;
    if (rc) return cuda_check(h, (cudaError_t)rc, "GlobalAveragePool");
    xn = t;
  }
  rc = gap_nhwc_launch(xn, (int)n, (int)c, (int)(hh * ww), y, h->stream);
  h->launches++;
  return rc ? cuda_check(h, (cudaError_t)rc, "GlobalAveragePool") : ONNXB200_OK;
}

// ---------------------------------------------------------------------------------- elementwise
int onnxb200_add(onnxb200_handle* h, const float* a, const int64_t* as, int ra, const float* b,
                 const int64_t* bs, int rb, int relu, float* y) {
  if (!h || !a || !b || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Add: null argument");
  cudaSetDevice(h->device);
  if (ra > 8 || rb > 8 || ra < 0 || rb < 0) return set_error(h, ONNXB200_ERR_UNSUPPORTED, "Add: rank > 8");
  // get_broadcast_shape (src/ops/tensor.rs:1536-1571)
  const int r = std::max(ra, rb);
  long long shape[8], sa[8], sb[8];
  long long total = 1;
  for (int i = 0; i < r; ++i) {
    const int64_t da = i >= r - ra ? as[i - (r - ra)] : 1;
    const int64_t db = i >= r - rb ? bs[i - (r - rb)] : 1;
    if (da != db && da != 1 && db != 1)
      return set_error(h, ONNXB200_ERR_VALIDATION, "Add: cannot broadcast shapes");
    shape[i] = da == 1 ? db : da;
    total *= shape[i];
  }
  long long ea = 1, eb = 1;
  for (int i = r - 1; i >= 0; --i) {
    const int64_t da = i >= r - ra ? as[i - (r - ra)] : 1;
    const int64_t db = i >= r - rb ? bs[i - (r - rb)] : 1;
    sa[i] = (da == 1) ? 0 : ea;
    sb[i] = (db == 1) ? 0 : eb;
    ea *= da;
    eb *= db;
  }
  if (r == 0) {
    shape[0] = 1;
    sa[0] = sb[0] = 0;
  }
  int rc = add_broadcast_launch(a, b, y, r == 0 ? 1 : r, shape, sa, sb, total, relu, h->stream);
  h->launches++;
  return rc ? cuda_check(h, (cudaError_t)rc, "Add") : ONNXB200_OK;
}

int onnxb200_relu(onnxb200_handle* h, const float* x, int64_t count, float* y) {
  if (!h || !x || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "Relu: null argument");
  cudaSetDevice(h->device);
  int rc = relu_launch(x, y, count, h->stream);
  h->launches++;
  return rc ? cuda_check(h, (cudaError_t)rc, "Relu") : ONNXB200_OK;
}

int onnxb200_batchnorm(onnxb200_handle* h, int layout, int64_t n, int64_t c, int64_t hh,
                       int64_t ww, const float* x, const float* scale, const float* bias,
                       const float* mean, const float* var, float eps, float* y) {
  if (!h || !x || !y || !scale || !bias || !mean || !var)
    return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "BatchNormalization: null argument");
  cudaSetDevice(h->device);
  int rc = ensure_workspace(h, 2 * align_up((size_t)c * 4));
  if (rc) return rc;
  float* s = static_cast<float*>(h->ws);
  float* t = reinterpret_cast<float*>(static_cast<uint8_t*>(h->ws) + align_up((size_t)c * 4));
  rc = bn_fold_launch(scale, bias, mean, var, nullptr, eps, (int)c, s, t, h->stream);
  h->launches++;
  if (rc) return cuda_check(h, (cudaError_t)rc, "BatchNormalization");
  if (layout == ONNXB200_LAYOUT_NHWC)
    rc = channel_affine_launch(x, s, t, y, n * hh * ww, (int)c, 1, 0, h->stream);
  else
    rc = channel_affine_launch(x, s, t, y, n, (int)c, hh * ww, 0, h->stream);
  h->launches++;
  return rc ? cuda_check(h, (cudaError_t)rc, "BatchNormalization") : ONNXB200_OK;
}

int onnxb200_nchw_to_nhwc(onnxb200_handle* h, int64_t n, int64_t c, int64_t hh, int64_t ww,
                          int64_t c_pad, const float* x, float* y) {
  if (!h || !x || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "repack: null argument");
  cudaSetDevice(h->device);
  if (c_pad < c) c_pad = c;
  int rc = nchw_to_nhwc_launch(x, (int)n, (int)c, (int)hh, (int)ww, (int)c_pad, y, h->stream);
  h->launches++;
  return rc ? cuda_check(h, (cudaError_t)rc, "NCHW->NHWC") : ONNXB200_OK;
}

int onnxb200_nhwc_to_nchw(onnxb200_handle* h, int64_t n, int64_t c, int64_t hh, int64_t ww,
                          const float* x, float* y) {
  if (!h || !x || !y) return set_error(h, ONNXB200_ERR_INVALID_ARGUMENT, "repack: null argument");
  cudaSetDevice(h->device);
  int rc = nhwc_to_nchw_launch(x, (int)n, (int)c, (int)hh, (int)ww, (int)c, y, h->stream);
  h->launches++;
  return rc ? cuda_check(h, (cudaError_t)rc, "NHWC->NCHW") : ONNXB200_OK;
}

}  // extern "C"
