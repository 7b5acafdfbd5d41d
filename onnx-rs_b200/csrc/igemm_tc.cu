// Host-side dispatch for the tcgen05 implicit-GEMM kernel (igemm_tc3.cu):
// tile-width choice, A-operand load mode, TMA maps of the A operand, and the
// alignment checks that turn a would-be misaligned launch into an error code.
//
// Replaces the reference's compute_conv2d_im2col + im2col_2d
// (src/ops/nn/conv.rs:1142-1368), its direct 1x1 path (conv.rs:849-935 via the
// SIMD strategy), compute_matmul's per-batch sgemm (src/ops/math/matmul.rs:124-279)
// and compute_gemm (src/ops/math/gemm.rs:172-291).
#include <algorithm>
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace ob2 {

namespace {
constexpr int kBM = 128;
}  // namespace

int igemm_pick_bn(const IgemmParams& p, int precision, int num_sms) {
  const int nc = p.Nc;
  if (nc <= 64) return 64;
  // Small problems (e.g. the late layers of a 32-image batch): 64-column tiles
  // when twice as many tiles still fit in one wave, so that more SMs work.
  const long long mt = (long long)((p.M + kBM - 1) / kBM) * p.batches;
  if (2 * mt * ((nc + 127) / 128) <= num_sms) return 64;
  // 3xTF32 (chunked accumulators, 3 x BN columns) and BF16 from fp32 activations
  // keep A slots in TMEM next to the accumulators: at most 128 columns wide.
  // TF32 and BF16 with bf16 activations and outputs keep only two whole-tile
  // accumulators, so 256 fits the 512 TMEM columns: twice the work per MMA
  // instruction (one thread issues them all) when there are enough tiles.
  const bool wide_ok = precision == kPrecTF32 || (precision == kPrecBF16 && p.a_bf16 && p.out_bf16 &&
                                                  p.num_kb > 2);
  if (!wide_ok) return 128;
  // Wide tiles halve A re-reads; use them when there are enough tiles to fill the GPU.
  if (nc >= 256 && mt * ((nc + 255) / 256) >= 2ll * num_sms) return 256;
  return 128;
}

IgemmParams second_source_view(const IgemmParams& p) {
  IgemmParams v = p;
  v.x = p.x2;
  v.Hin = p.H2;
  v.Win = p.W2;
  v.Cs = p.Cs2;
  v.KW = 1;
  v.sh = v.sw = p.s2;
  v.ph = v.pw = 0;
  v.dh = v.dw = 1;
  v.K = p.Cs2;
  v.a_mode = p.a_mode2;
  v.kb_split = 0;
  return v;
}

int igemm_launch(const IgemmParams& p, const CUtensorMap& hi, const CUtensorMap& lo,
                 const CUtensorMap& am, const CUtensorMap& am2, int precision, int bn, int num_sms,
                 cudaStream_t st) {
  if (p.a_mode != kALoadGather &&
      (p.a_mode == kALoadIm2colTaps ? ((p.Cs != 4 && p.Cs != 8 && p.Cs != 16) || p.K % p.Cs != 0)
       : p.a_mode == kALoadIm2col   ? p.Cs % 32 != 0
                                    : p.Cs < 32))
    return (int)cudaErrorInvalidValue;
  // The kernel moves 16-byte vectors: refuse (instead of faulting on) any
  // pointer or stride that would make one of them misaligned.
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (!p.x || !p.y || mis(p.x) || mis(p.y) || (p.res && mis(p.res)) || (p.scale && mis(p.scale)) ||
      (p.shift && mis(p.shift)) || p.Cs % 4 || p.Nc % 4 || p.ldy % 4 || (p.res && p.ldr % 4) ||
      p.y_bstride % 4 || p.num_kb <= 0 || (p.batches > 1 && p.ksplit <= 1 && !p.a_off && p.M % 4))
    return (int)cudaErrorMisalignedAddress;
  // two sources: source 1 a [pixels][Cs] matrix of whole k-blocks, source 2 a
  // 1x1 convolution of whole k-blocks at the same output pixels
  const int bk = igemm_block_k(precision, p.a_bf16 != 0);
  // bf16 activations: whole taps per k-block through TMA, no padding
  if (p.a_bf16 && (p.a_mode == kALoadGather || p.a_mode == kALoadIm2colTaps || p.Cs % bk || p.K % bk))
    return (int)cudaErrorInvalidValue;
  // K split: `ksplit` batches over one A and B, whole k-blocks per slice
  if (p.ksplit > 1 && (p.batches != p.ksplit || p.a_off || p.b_row || p.res || p.scale || p.shift ||
                       p.relu || p.out_bf16 || p.num_kb % p.ksplit))
    return (int)cudaErrorInvalidValue;
  if (p.kb_split &&
      (p.a_mode != kALoadTma2d || p.Cs != p.kb_split * bk || p.batches != (p.ksplit > 1 ? p.ksplit : 1) ||
       p.a_off || !p.x2 ||
       mis(p.x2) || p.Cs2 % bk || p.s2 < 1 || p.num_kb != p.kb_split + p.Cs2 / bk ||
       (p.a_mode2 != kALoadTma2d && p.a_mode2 != kALoadIm2col) ||
       (p.a_mode2 == kALoadTma2d && (p.s2 != 1 || p.H2 != p.OH || p.W2 != p.OW))))
    return (int)cudaErrorInvalidValue;
  if (precision == kPrec3xTF32 || precision == kPrecTF32 || precision == kPrecBF16)
    return igemm3_launch(p, hi, lo, am, am2, precision, bn, num_sms, st);
  return (int)cudaErrorInvalidValue;
}

int igemm_launch_split(const IgemmParams& p, int ksplit, int split_mt, float* ws, const CUtensorMap& hi,
                       const CUtensorMap& lo, const CUtensorMap& am, const CUtensorMap& am2, int precision,
                       int bn, int num_sms, cudaStream_t st) {
  if (ksplit <= 1) return igemm_launch(p, hi, lo, am, am2, precision, bn, num_sms, st);
  const int m_tiles = (p.M + kBM - 1) / kBM;
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 15) || p.batches != 1 || p.a_off || p.b_row || p.a_bf16 ||
      p.out_bf16 || p.num_kb % ksplit || p.m_base || split_mt < 0 || split_mt >= m_tiles)
    return (int)cudaErrorInvalidValue;
  int rc = 0;
  const int m0 = split_mt * kBM;
  if (split_mt > 0) {  // the whole waves of tiles, unsplit, with the full epilogue
    IgemmParams h = p;
    h.M = m0;
    h.m_tiles = split_mt;
    rc = igemm_launch(h, hi, lo, am, am2, precision, bn, num_sms, st);
    if (rc) return rc;
  }
  // the tail rows [m0, M): slice b's raw sums -> ws[b][M - m0][Nc]
  const int mt_rows = p.M - m0;
  IgemmParams q = p;
  q.m_base = m0;
  q.M = mt_rows;
  q.m_tiles = m_tiles - split_mt;
  q.ksplit = ksplit;
  q.batches = ksplit;
  q.y = ws;
  q.ldy = p.Nc;
  q.y_bstride = (long long)mt_rows * p.Nc;
  q.scale = q.shift = q.res = nullptr;
  q.relu = 0;
  q.out_bf16 = 0;
  rc = igemm_launch(q, hi, lo, am, am2, precision, bn, num_sms, st);
  if (rc) return rc;
  return splitk_reduce_launch(ws, ksplit, mt_rows, p.Nc, p.y + (long long)m0 * p.ldy, p.ldy, p.scale, p.shift,
                              p.res ? p.res + (long long)m0 * p.ldr : nullptr, p.ldr, p.relu, st);
}

void igemm_pick_split(const IgemmParams& p, bool residual, int precision, int num_sms, int* bn, int* ksplit,
                      int* split_mt) {
  const int bn0 = igemm_pick_bn(p, precision, num_sms);
  *bn = bn0;
  *ksplit = 1;
  *split_mt = 0;
  if (p.batches != 1 || p.a_off || p.b_row || p.a_bf16 || p.out_bf16 || p.num_kb < 8 || num_sms <= 0) return;
  // modelled time in units of one k-block of a 128-column tile; a 64-column
  // tile's k-block costs ~0.8 of it (its MMAs are half as long, the operand
  // round trip is not)
  const double kb_us = precision == kPrec3xTF32 ? 0.8 : 0.5;
  const long long mt = (p.M + kBM - 1) / kBM;
  // M-tiles [m_from, m_to) with tile width b, K split s (1 = none)
  auto cost = [&](int b, int s, long long m_from, long long m_to) {
    const long long tiles = (m_to - m_from) * ((p.Nc + b - 1) / b);
    const long long waves = (tiles * s + num_sms - 1) / num_sms;
    double c = (double)waves * (p.num_kb / s) * (b == 64 ? 0.8 : 1.0);
    if (s > 1) {  // reduction pass: read the s slices (from L2 when they fit it,
                  // ~10 TB/s), read the residual and write y from / to HBM (~6 TB/s)
      const double rows = (double)std::min<long long>(p.M, m_to * kBM) - (double)(m_from * kBM);
      const double slice = rows * p.Nc * 4.0;
      const double ws_gbs = s * slice <= 64e6 ? 10.0e6 : 6.0e6;  // bytes per us
      c += (s * slice / ws_gbs + (1 + (residual ? 1 : 0)) * slice / 6.0e6 + 2.0) / kb_us;
    }
    return c;
  };
  const double unsplit = cost(bn0, 1, 0, mt);
  double best = unsplit;
  int best_bn = bn0, best_s = 1, best_mt = 0;
  const int cands[2] = {bn0, (bn0 == 64 && p.Nc > 64 && precision != kPrecTF32) ? 128 : 0};
  for (int b : cands) {
    if (!b) continue;
    const long long nt = (p.Nc + b - 1) / b;
    // tail split: the whole waves of tiles (whole M-tiles of them) unsplit, the
    // remaining M-tiles split, in a second launch (+~3 us)
    const long long full = (mt * nt) / num_sms * num_sms;
    const long long mt0 = full / nt;
    for (int s = 2; s <= 16; ++s) {
      if (p.num_kb % s || p.num_kb / s < 4) continue;
      const double c_all = cost(b, s, 0, mt);
      if (c_all < best) {
        best = c_all;
        best_bn = b;
        best_s = s;
        best_mt = 0;
      }
      if (mt0 > 0 && mt0 < mt) {
        const double c_tail = cost(b, 1, 0, mt0) + cost(b, s, mt0, mt) + 3.0 / kb_us;
        if (c_tail < best) {
          best = c_tail;
          best_bn = b;
          best_s = s;
          best_mt = (int)mt0;
        }
      }
    }
  }
  if (best_s > 1 && best < 0.94 * unsplit) {
    *bn = best_bn;
    *ksplit = best_s;
    *split_mt = best_mt;
  }
}

int pick_a_mode(const IgemmParams& p, int precision) {
  // A k-block is 32 fp32 (one 128-byte TMA row per pixel): 32 channels of one
  // filter tap, or 32 / Cs whole taps of a 4-, 8- or 16-channel tensor.  With
  // bf16 activations it is 64 channels of one tap, TMA only (Cs % 64 == 0).
  const bool single_tap = p.K == p.Cs;
  if (p.a_bf16) {
    if (p.Cs % 64) return kALoadGather;  // refused by igemm_launch
    if (single_tap && p.sh == 1 && p.sw == 1 && p.ph == 0 && p.pw == 0 && p.OH == p.Hin && p.OW == p.Win)
      return kALoadTma2d;
  }
  if (single_tap && p.sh == 1 && p.sw == 1 && p.ph == 0 && p.pw == 0 && p.OH == p.Hin &&
      p.OW == p.Win)  // rows of A are rows of the [pixels][channels] matrix; the
                      // box of the last k-block may run past Cs (zero fill)
    return p.Cs >= 32 ? kALoadTma2d : kALoadGather;
  const bool few_ch = (p.Cs == 4 || p.Cs == 8 || p.Cs == 16) && p.K % p.Cs == 0;
  if (!few_ch && p.Cs % 32 != 0) return kALoadGather;
  // im2col maps: 4-D corners are 8-bit signed, the filter-tap offsets 8-bit
  // unsigned (small convolutions always fit); one image batch per launch.
  if (p.batches != 1 || p.a_off) return kALoadGather;
  const int up_w = (p.OW - 1) * p.sw - p.pw - (p.Win - 1);
  const int up_h = (p.OH - 1) * p.sh - p.ph - (p.Hin - 1);
  const int taps = p.K / p.Cs;
  const int kh = (taps + p.KW - 1) / p.KW;
  if (p.pw > 127 || p.ph > 127 || up_w < -128 || up_h < -128 || up_w > 127 || up_h > 127 ||
      (p.KW - 1) * p.dw > 255 || (kh - 1) * p.dh > 255 || p.sw > 8 || p.sh > 8)
    return kALoadGather;
  return few_ch ? kALoadIm2colTaps : kALoadIm2col;
}

namespace {
typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
typedef CUresult (*EncodeIm2colFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const int*, const int*,
                                   cuuint32_t, cuuint32_t, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
void* driver_fn(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return fn;
}
}  // namespace

int encode_a_map(const IgemmParams& p, int n, CUtensorMap* map) {
  void* base = const_cast<float*>(p.x);
  const int esz_a = p.a_bf16 ? 2 : 4;
  if (p.a_mode == kALoadTma2d) {
    static EncodeTiledFn2 fn = reinterpret_cast<EncodeTiledFn2>(driver_fn("cuTensorMapEncodeTiled"));
    if (!fn) return (int)CUDA_ERROR_NOT_FOUND;
    // n = number of rows of the [rows][Cs] matrix (pixels of the batch, or all A rows)
    const int esz = p.a_bf16 ? 2 : 4;
    cuuint64_t dims[2] = {(cuuint64_t)p.Cs, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)p.Cs * esz};
    cuuint32_t box[2] = {p.a_bf16 ? 64u : 32u, (cuuint32_t)kBM};
    cuuint32_t es[2] = {1u, 1u};
    return (int)fn(map, p.a_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base,
                   dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  static EncodeIm2colFn fn = reinterpret_cast<EncodeIm2colFn>(driver_fn("cuTensorMapEncodeIm2col"));
  if (!fn) return (int)CUDA_ERROR_NOT_FOUND;
  // NHWC tensor, dims innermost first: C, W, H, N (n = images)
  cuuint64_t dims[4] = {(cuuint64_t)p.Cs, (cuuint64_t)p.Win, (cuuint64_t)p.Hin, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)p.Cs * esz_a, (cuuint64_t)p.Win * p.Cs * esz_a,
                           (cuuint64_t)p.Hin * p.Win * p.Cs * esz_a};
  // Bounding box of the base (top-left) input pixel of every output pixel:
  // W from -pw to (OW-1)*sw - pw, H likewise; traversal stride = conv stride.
  int lower[2] = {-p.pw, -p.ph};
  int upper[2] = {(p.OW - 1) * p.sw - p.pw - (p.Win - 1), (p.OH - 1) * p.sh - p.ph - (p.Hin - 1)};
  cuuint32_t es[4] = {1u, (cuuint32_t)p.sw, (cuuint32_t)p.sh, 1u};
  // taps mode: one box = all Cs channels (16 to 64 bytes) of 128 pixels for one
  // tap, unswizzled; otherwise 32 channels in 128-byte swizzled rows
  const bool taps = p.a_mode == kALoadIm2colTaps;
  return (int)fn(map, p.a_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base,
                 dims, strides, lower, upper, taps ? (cuuint32_t)p.Cs : (p.a_bf16 ? 64u : 32u),
                 (cuuint32_t)kBM, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 taps ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace ob2
