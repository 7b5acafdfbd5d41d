// CUDA-core kernels of the path: grouped / general direct convolution, a
// fallback batched GEMM, weight packing for the tcgen05 kernel, layout
// repacks, MaxPool, GlobalAveragePool and elementwise ops.  All memory-bound
// kernels move 16-byte vectors along the channel (innermost NHWC) axis.
#include <algorithm>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace ob2 {

namespace {
constexpr int kBlock = 256;

inline int grid_for(long long n, int block) {
  long long g = (n + block - 1) / block;
  if (g > (1ll << 30)) g = 1ll << 30;
  return (int)(g < 1 ? 1 : g);
}

__device__ __forceinline__ float epi(float v, const float* scale, const float* shift, int c) {
  if (scale) v *= scale[c];
  if (shift) v += shift[c];
  return v;
}
}  // namespace

// ------------------------------------------------------------------ direct conv
// compute_conv2d_direct_impl (src/ops/nn/conv.rs:849-935) on NHWC data: one
// thread per output element (n, oh, ow, co) with co fastest; sums over
// (ci, kh, kw) of its group in fp32.
__global__ void conv_direct_kernel(const float* __restrict__ x, int N, int H, int W, int C,
                                   int Cs, const float* __restrict__ w, int CO, int KH, int KW, int sh,
                                   int sw, int ph, int pw, int dh, int dw, int group, int OH,
                                   int OW, const float* __restrict__ scale,
                                   const float* __restrict__ shift, const float* __restrict__ res,
                                   int relu, float* __restrict__ y) {
  const long long total = (long long)N * OH * OW * CO;
  const int cg = C / group, cog = CO / group;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int co = (int)(idx % CO);
    long long pix = idx / CO;
    const int ow = (int)(pix % OW);
    const int oh = (int)((pix / OW) % OH);
    const int n = (int)(pix / ((long long)OW * OH));
    const int g = co / cog;
    float sum = 0.f;
    for (int ci = 0; ci < cg; ++ci) {
      const float* wp = w + ((long long)co * cg + ci) * KH * KW;
      for (int r = 0; r < KH; ++r) {
        const int ih = oh * sh - ph + r * dh;
        if ((unsigned)ih >= (unsigned)H) continue;
        for (int s = 0; s < KW; ++s) {
          const int iw = ow * sw - pw + s * dw;
          if ((unsigned)iw >= (unsigned)W) continue;
          sum = fmaf(x[(((long long)n * H + ih) * W + iw) * Cs + g * cg + ci], wp[r * KW + s], sum);
        }
      }
    }
    float v = epi(sum, scale, shift, co);
    if (res) v += res[idx];
    if (relu) v = v > 0.f ? v : 0.f;
    y[idx] = v;
  }
}

// Grouped convolution with 4-aligned group widths (e.g. ResNeXt's 32 groups of
// 4 channels): one thread per (output pixel, 4 output channels of one group),
// 16-byte input and output vectors, the OIHW weights staged in shared memory as
// [tap][ci][co] (the lanes of a warp hold consecutive output-channel quadruples
// of one pixel and read one 16-byte weight vector each).  KH, KW, CG4 = cg / 4
// are compile-time (0 = runtime) so that a 3x3 filter's loads are all issued
// before its FMAs.  Sums over (kh, kw, ci) in fp32.
template <int KH_, int KW_, int CG4_>
__global__ void conv_grouped_v4_kernel(const float* __restrict__ x, int H, int W, int Cs,
                                       const float* __restrict__ w, int CO, int cg_rt, int cog,
                                       int KH_rt, int KW_rt, int sh, int sw, int ph, int pw, int dh,
                                       int dw, int OH, int OW, long long total4,
                                       const float* __restrict__ scale,
                                       const float* __restrict__ shift, const float* __restrict__ res,
                                       int relu, float* __restrict__ y) {
  const int KH = KH_ ? KH_ : KH_rt, KW = KW_ ? KW_ : KW_rt, cg = CG4_ ? 4 * CG4_ : cg_rt;
  extern __shared__ float ws[];
  const int wn = CO * cg * KH * KW;
  for (int i = threadIdx.x; i < wn; i += blockDim.x) {  // i = (tap*cg + ci)*CO + co
    const int co = i % CO, tc = i / CO;
    const int ci = tc % cg, tap = tc / cg;
    ws[i] = __ldg(w + ((long long)co * cg + ci) * (KH * KW) + tap);
  }
  __syncthreads();
  const unsigned CO4 = CO / 4;
  // 32-bit index math (the launcher guarantees total4 < 2^31): 64-bit divisions
  // would dominate the cost of this kernel
  for (unsigned idx = blockIdx.x * blockDim.x + threadIdx.x; idx < (unsigned)total4;
       idx += gridDim.x * blockDim.x) {
    const int co0 = (int)(idx % CO4) * 4;
    const unsigned pix = idx / CO4;
    const int ow = (int)(pix % (unsigned)OW);
    const unsigned t = pix / (unsigned)OW;
    const int oh = (int)(t % (unsigned)OH);
    const long long n = t / (unsigned)OH;
    const int cin0 = (co0 / cog) * cg;
    const float* xb = x + n * H * W * Cs + cin0;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (KH_ > 0 && KW_ > 0 && CG4_ > 0) {
      float4 xin[KH_ * KW_][CG4_];
#pragma unroll
      for (int r = 0; r < KH_; ++r)
#pragma unroll
        for (int q = 0; q < KW_; ++q) {
          const int ih = oh * sh - ph + r * dh, iw = ow * sw - pw + q * dw;
          const bool in = (unsigned)ih < (unsigned)H && (unsigned)iw < (unsigned)W;
          const float4* xp = reinterpret_cast<const float4*>(xb + ((long long)ih * W + iw) * Cs);
#pragma unroll
          for (int c4 = 0; c4 < CG4_; ++c4)
            xin[r * KW_ + q][c4] = in ? __ldg(xp + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int tap = 0; tap < KH_ * KW_; ++tap)
#pragma unroll
        for (int c4 = 0; c4 < CG4_; ++c4) {
          const float xs[4] = {xin[tap][c4].x, xin[tap][c4].y, xin[tap][c4].z, xin[tap][c4].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 wv = *reinterpret_cast<const float4*>(ws + (tap * cg + 4 * c4 + e) * CO + co0);
            acc[0] = fmaf(xs[e], wv.x, acc[0]);
            acc[1] = fmaf(xs[e], wv.y, acc[1]);
            acc[2] = fmaf(xs[e], wv.z, acc[2]);
            acc[3] = fmaf(xs[e], wv.w, acc[3]);
          }
        }
    } else {
      for (int r = 0; r < KH; ++r) {
        const int ih = oh * sh - ph + r * dh;
        if ((unsigned)ih >= (unsigned)H) continue;
        for (int q = 0; q < KW; ++q) {
          const int iw = ow * sw - pw + q * dw;
          if ((unsigned)iw >= (unsigned)W) continue;
          const float4* xp = reinterpret_cast<const float4*>(xb + ((long long)ih * W + iw) * Cs);
          const float* wt = ws + (r * KW + q) * cg * CO + co0;
          for (int c4 = 0; c4 < cg / 4; ++c4) {
            const float4 xv = __ldg(xp + c4);
            const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float4 wv = *reinterpret_cast<const float4*>(wt + (4 * c4 + e) * CO);
              acc[0] = fmaf(xs[e], wv.x, acc[0]);
              acc[1] = fmaf(xs[e], wv.y, acc[1]);
              acc[2] = fmaf(xs[e], wv.z, acc[2]);
              acc[3] = fmaf(xs[e], wv.w, acc[3]);
            }
          }
        }
      }
    }
    const long long o = (long long)pix * CO + co0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v = epi(acc[j], scale, shift, co0 + j);
      if (res) v += res[o + j];
      if (relu) v = v > 0.f ? v : 0.f;
      acc[j] = v;
    }
    *reinterpret_cast<float4*>(y + o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
}

// Grouped 3x3 convolution (dilation 1, stride S) over output-row segments: a
// thread computes P consecutive output pixels of one row for 4 output channels
// of one group.  Per filter row and input-channel quadruple it loads the
// (P-1)*S+3 input vectors its segment touches once into registers, then for
// each of the 3 taps and 4 channels reads one 16-byte weight vector from shared
// memory and applies it to all P pixels (4P FMAs per shared-memory load; the
// per-pixel kernel above does 4).  A block works on one slice of CB output
// channels and keeps only that slice's weights, [tap][ci][co in slice], in
// shared memory, so that wide groups (e.g. 32 groups of 32 channels) fit.
// Sums over (kh, ci, kw) in fp32.
template <int S, int P>
__global__ void __launch_bounds__(256, 2)
    conv_grouped_row_kernel(const float* __restrict__ x, int H, int W, int Cs,
                            const float* __restrict__ w, int CB, int CO, int cg, int cog, int ph,
                            int pw, int OH, int OW, int nseg, unsigned per_slice,
                            int blocks_per_slice, const float* __restrict__ scale,
                            const float* __restrict__ shift, const float* __restrict__ res, int relu,
                            float* __restrict__ y) {
  extern __shared__ float ws[];
  const int slice = blockIdx.x / blocks_per_slice, bis = blockIdx.x % blocks_per_slice;
  const int cb0 = slice * CB;
  // the slice's OIHW weights are one contiguous run: each thread copies whole
  // 9-tap filters (coalesced across the warp) into the [tap][ci][co] layout
  const float* wsl = w + (long long)cb0 * cg * 9;
  for (int j = threadIdx.x; j < CB * cg; j += blockDim.x) {
    const int c = j / cg, ci = j - c * cg;
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) ws[(tap * cg + ci) * CB + c] = __ldg(wsl + j * 9 + tap);
  }
  __syncthreads();
  constexpr int NI = (P - 1) * S + 3;
  const unsigned CB4 = CB / 4;
  const int Cs4 = Cs / 4;
  for (unsigned idx = bis * blockDim.x + threadIdx.x; idx < per_slice;
       idx += blocks_per_slice * blockDim.x) {
    const int c0 = (int)(idx % CB4) * 4;
    unsigned t = idx / CB4;
    const int seg = (int)(t % (unsigned)nseg);
    t /= (unsigned)nseg;
    const int oh = (int)(t % (unsigned)OH);
    const unsigned n = t / (unsigned)OH;
    const int co0 = cb0 + c0;
    const int ow0 = seg * P, iw0 = ow0 * S - pw;
    const float4* xb = reinterpret_cast<const float4*>(x + (size_t)n * H * W * Cs + (co0 / cog) * cg);
    float acc[P][4];
#pragma unroll
    for (int p = 0; p < P; ++p) acc[p][0] = acc[p][1] = acc[p][2] = acc[p][3] = 0.f;
    // the lanes of a warp usually share one row segment, so these branches are uniform
    const bool interior = iw0 >= 0 && iw0 + NI <= W;
    for (int c4 = 0; c4 < cg / 4; ++c4) {
      for (int r = 0; r < 3; ++r) {
        const int ih = oh * S - ph + r;
        if ((unsigned)ih >= (unsigned)H) continue;  // zero rows add nothing
        const float4* xrow = xb + ((size_t)ih * W + iw0) * Cs4 + c4;
        float4 xin[NI];
        if (interior) {
#pragma unroll
          for (int i = 0; i < NI; ++i) xin[i] = __ldg(xrow + i * Cs4);
        } else {
#pragma unroll
          for (int i = 0; i < NI; ++i)
            xin[i] = (unsigned)(iw0 + i) < (unsigned)W ? __ldg(xrow + i * Cs4)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float* wr = ws + (r * 3 * cg + 4 * c4) * CB + c0;
#pragma unroll
        for (int q = 0; q < 3; ++q)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 wv = *reinterpret_cast<const float4*>(wr + (q * cg + e) * CB);
#pragma unroll
            for (int p = 0; p < P; ++p) {
              const float4 xv = xin[p * S + q];
              const float xs = e == 0 ? xv.x : e == 1 ? xv.y : e == 2 ? xv.z : xv.w;
              acc[p][0] = fmaf(xs, wv.x, acc[p][0]);
              acc[p][1] = fmaf(xs, wv.y, acc[p][1]);
              acc[p][2] = fmaf(xs, wv.z, acc[p][2]);
              acc[p][3] = fmaf(xs, wv.w, acc[p][3]);
            }
          }
      }
    }
    // epilogue: y = acc * scale + shift (+ res) (Relu), 16-byte vectors
    const float4 sc = scale ? __ldg(reinterpret_cast<const float4*>(scale + co0)) : make_float4(1.f, 1.f, 1.f, 1.f);
    const float4 sf = shift ? __ldg(reinterpret_cast<const float4*>(shift + co0)) : make_float4(0.f, 0.f, 0.f, 0.f);
    const long long o0 = (((long long)n * OH + oh) * OW + ow0) * CO + co0;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      if (ow0 + p >= OW) break;
      const long long o = o0 + (long long)p * CO;
      float4 v = make_float4(fmaf(acc[p][0], sc.x, sf.x), fmaf(acc[p][1], sc.y, sf.y),
                             fmaf(acc[p][2], sc.z, sf.z), fmaf(acc[p][3], sc.w, sf.w));
      if (res) {
        const float4 rv = __ldg(reinterpret_cast<const float4*>(res + o));
        v.x += rv.x, v.y += rv.y, v.z += rv.z, v.w += rv.w;
      }
      if (relu) v = make_float4(fmaxf(v.x, 0.f), fmaxf(v.y, 0.f), fmaxf(v.z, 0.f), fmaxf(v.w, 0.f));
      *reinterpret_cast<float4*>(y + o) = v;
    }
  }
}

namespace {
// Output-channel slice of the row kernel: the widest divisor of CO that is a
// multiple of 4 and whose [tap][ci][co] weights fit 64 KB of shared memory.
int grouped_row_slice(int CO, int cg) {
  const long long per_co = (long long)cg * 9 * sizeof(float);
  for (int cb = CO; cb >= 4; --cb)
    if (CO % cb == 0 && cb % 4 == 0 && cb * per_co <= 64 * 1024) return cb;
  return 0;
}
}  // namespace

// ------------------------------------------------------------ K-split reduction
// y[m][n] = relu(sum_s ws[s][m][n] * scale[n] + shift[n] + res[m][n]), slices
// summed in order; one thread per 4 consecutive columns (16-byte vectors).
__global__ void splitk_reduce_kernel(const float4* __restrict__ ws, int S, long long MN4, int N4,
                                     float* __restrict__ y, int ldy, const float* __restrict__ scale,
                                     const float* __restrict__ shift, const float* __restrict__ res, int ldr,
                                     int relu) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < MN4;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / N4;
    const int n = (int)(i - m * N4) * 4;
    float4 a = __ldg(ws + i);
    for (int sl = 1; sl < S; ++sl) {
      const float4 b = __ldg(ws + sl * MN4 + i);
      a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
    }
    if (scale) {
      const float4 sc = __ldg(reinterpret_cast<const float4*>(scale + n));
      a.x *= sc.x, a.y *= sc.y, a.z *= sc.z, a.w *= sc.w;
    }
    if (shift) {
      const float4 sh = __ldg(reinterpret_cast<const float4*>(shift + n));
      a.x += sh.x, a.y += sh.y, a.z += sh.z, a.w += sh.w;
    }
    if (res) {
      const float4 rv = __ldg(reinterpret_cast<const float4*>(res + m * ldr + n));
      a.x += rv.x, a.y += rv.y, a.z += rv.z, a.w += rv.w;
    }
    if (relu) a = make_float4(fmaxf(a.x, 0.f), fmaxf(a.y, 0.f), fmaxf(a.z, 0.f), fmaxf(a.w, 0.f));
    *reinterpret_cast<float4*>(y + m * ldy + n) = a;
  }
}

int splitk_reduce_launch(const float* ws, int ksplit, int M, int N, float* y, int ldy, const float* scale,
                         const float* shift, const float* res, int ldr, int relu, cudaStream_t st) {
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (ksplit < 1 || N % 4 || ldy % 4 || (res && ldr % 4) || !ws || !y || mis(ws) || mis(y) ||
      (scale && mis(scale)) || (shift && mis(shift)) || (res && mis(res)))
    return (int)cudaErrorMisalignedAddress;
  const long long mn4 = (long long)M * N / 4;
  if (mn4 == 0) return 0;
  const int blocks = (int)std::min<long long>((mn4 + kBlock - 1) / kBlock, 148LL * 16);
  splitk_reduce_kernel<<<blocks, kBlock, 0, st>>>(reinterpret_cast<const float4*>(ws), ksplit, mn4, N / 4, y,
                                                  ldy, scale, shift, res, ldr, relu);
  return (int)cudaGetLastError();
}

int conv_simt_igemm_launch(const float* x, int N, int H, int W, int C, int Cs, const float* w, int CO,
                           int KH, int KW, int sh, int sw, int ph, int pw, int dh, int dw, int OH, int OW,
                           const float* scale, const float* shift, const float* res, int relu, float* y,
                           cudaStream_t st);

int conv_direct_launch(const float* x, int N, int H, int W, int C, int Cs, const float* w, int CO,
                       int KH, int KW, int sh, int sw, int ph, int pw, int dh, int dw, int group, int OH,
                       int OW, const float* scale, const float* shift, const float* res, int relu,
                       float* y, cudaStream_t st) {
  const long long total = (long long)N * OH * OW * CO;
  if (total == 0) return 0;
  const int cg = C / group, cog = CO / group;
  const size_t wbytes = (size_t)CO * cg * KH * KW * sizeof(float);
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool al = a16(x) && a16(y) && (!res || a16(res)) && (!scale || a16(scale)) &&
                  (!shift || a16(shift));
  // 3x3 stride 1 / 2 (ResNeXt's grouped convolutions): row segments of 7 pixels
  constexpr int kSeg = 7;
  if (group > 1 && KH == 3 && KW == 3 && dh == 1 && dw == 1 && sh == sw && (sh == 1 || sh == 2) &&
      cg % 4 == 0 && cog % 4 == 0 && Cs % 4 == 0 && al) {
    const int CB = grouped_row_slice(CO, cg);
    const int nseg = (OW + kSeg - 1) / kSeg;
    const long long per_slice = (long long)N * OH * nseg * (CB / 4);
    if (CB > 0 && per_slice < (1ll << 31) && (long long)N * H * W * Cs < (1ll << 40)) {
      const int nslices = CO / CB;
      // persistent: one wave of resident blocks in all, each staging its
      // slice's weights once
      auto kern = sh == 1 ? conv_grouped_row_kernel<1, kSeg> : conv_grouped_row_kernel<2, kSeg>;
      static int resident[2] = {0, 0};  // blocks per SM (same for every B200)
      int& occ = resident[sh - 1];
      const size_t sbytes = (size_t)CB * cg * 9 * sizeof(float);
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024) != cudaSuccess)
        return (int)cudaGetLastError();
      if (!occ && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, 64 * 1024) != cudaSuccess)
        return (int)cudaGetLastError();
      int sms = 148, dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const int bps = (int)std::max<long long>(
          1, std::min<long long>((per_slice + 255) / 256,
                                 ((long long)sms * std::max(occ, 1) + nslices - 1) / nslices));
      kern<<<nslices * bps, 256, sbytes, st>>>(x, H, W, Cs, w, CB, CO, cg, cog, ph, pw, OH, OW, nseg,
                                               (unsigned)per_slice, bps, scale, shift, res, relu, y);
      return (int)cudaGetLastError();
    }
  }
  if (group > 1 && cg % 4 == 0 && cog % 4 == 0 && Cs % 4 == 0 && wbytes <= 96 * 1024 && a16(x) &&
      a16(y) && (!res || a16(res)) && total / 4 < (1ll << 31)) {
    const long long total4 = total / 4;
    const int blocks = (int)std::min<long long>((total4 + 255) / 256, 148LL * 4);
    auto go = [&](auto kern) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      kern<<<blocks, 256, wbytes, st>>>(x, H, W, Cs, w, CO, cg, cog, KH, KW, sh, sw, ph, pw, dh, dw,
                                        OH, OW, total4, scale, shift, res, relu, y);
    };
    if (KH == 3 && KW == 3 && cg == 4) go(conv_grouped_v4_kernel<3, 3, 1>);
    else if (KH == 3 && KW == 3 && cg == 8) go(conv_grouped_v4_kernel<3, 3, 2>);
    else go(conv_grouped_v4_kernel<0, 0, 0>);
    return (int)cudaGetLastError();
  }
  // ungrouped (the fp32 precision mode): implicit GEMM on the CUDA cores
  const long long npix = (long long)N * OH * OW;
  if (group == 1 && (npix + 127) / 128 <= 65535 && (long long)C * KH * KW < (1ll << 31))
    return conv_simt_igemm_launch(x, N, H, W, C, Cs, w, CO, KH, KW, sh, sw, ph, pw, dh, dw, OH, OW,
                                  scale, shift, res, relu, y, st);
  conv_direct_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(
      x, N, H, W, C, Cs, w, CO, KH, KW, sh, sw, ph, pw, dh, dw, group, OH, OW, scale, shift, res,
      relu, y);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ SIMT GEMM
// fp32 FFMA GEMM for the exact-fp32 precision mode and for shapes the tensor-core
// path refuses.  A 256-thread block owns a 128 x 128 output tile; a thread owns
// 8 x 8 outputs as two 4-row groups 64 rows apart times two 4-column groups 64
// columns apart, so that a warp's shared-memory reads are conflict-free 16-byte
// vectors.  K advances 8 at a time: the next step's A and B tiles are read into
// registers (16-byte global loads where the operand's pointer and leading
// dimension allow) while the current step's tiles are multiplied from the other
// shared-memory buffer.  Every output sums its K products in order, k = 0, 1, ...,
// with fmaf.  With kConv the A operand is an ungrouped NHWC convolution's input
// gathered on the fly (implicit GEMM): row m = output pixel (n, oh, ow), column
// k = (ci, r, s) in the order of the OIHW weights, which are B as stored
// ([c_out][k], trans_b); padding taps read as 0.
constexpr int kSgBM = 128, kSgBN = 128, kSgBK = 8;

struct SimtConvGeom {
  int H, W, Cs, OH, OW, KH, KW, sh, sw, ph, pw, dh, dw;
};

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

template <bool kConv>
__global__ void __launch_bounds__(256, 2)
gemm_simt_kernel(const float* __restrict__ a, const float* __restrict__ b, const long long* a_off,
                 const long long* b_off, long long y_bstride, int M, int N, int K, int lda, int ldb,
                 int ta, int tb, const float* __restrict__ scale, const float* __restrict__ shift,
                 const float* __restrict__ res, int ldr, int relu, float* __restrict__ y, int ldy,
                 SimtConvGeom g) {
  __shared__ __align__(16) float As[2][kSgBK][kSgBM];
  __shared__ __align__(16) float Bs[2][kSgBK][kSgBN];
  const int bz = blockIdx.z;
  const float* A = a + (a_off ? a_off[bz] : 0);
  const float* B = b + (b_off ? b_off[bz] : 0);
  float* Y = y + (long long)bz * y_bstride;
  const float* R = res ? res + (long long)bz * y_bstride : nullptr;
  const int m0 = blockIdx.y * kSgBM, n0 = blockIdx.x * kSgBN;
  const int t = threadIdx.x, tx = t % 16, ty = t / 16;
  const bool va = (lda & 3) == 0 && aligned16(A);
  const bool vb = (ldb & 3) == 0 && aligned16(B);
  // This thread's share of a K step: four A values and four B values, either
  // four consecutive k of one row (operand stored with k contiguous) or one k of
  // four consecutive rows (operand stored with rows contiguous).
  const int a_r = ta ? (t % 32) * 4 : t / 2, a_k = ta ? t / 32 : (t % 2) * 4;
  const int b_r = tb ? t / 2 : (t % 32) * 4, b_k = tb ? (t % 2) * 4 : t / 32;
  // kConv: this thread's output pixel, its filter window origin and its image
  const float* cx = A;
  int cih0 = 0, ciw0 = 0;
  bool cok = false;
  if constexpr (kConv) {
    const int m = m0 + a_r;
    cok = m < M;
    if (cok) {
      const int ow = m % g.OW, q = m / g.OW, oh = q % g.OH, n = q / g.OH;
      cih0 = oh * g.sh - g.ph;
      ciw0 = ow * g.sw - g.pw;
      cx = A + (long long)n * g.H * g.W * g.Cs;
    }
  }
  float ra[4], rb[4];
  auto load = [&](int k0) {
    if constexpr (kConv) {  // four consecutive (ci, r, s) of this thread's pixel
      const int k = k0 + a_k, khw = g.KH * g.KW;
      int ci = k / khw, rs = k - ci * khw;
      int r = rs / g.KW, s = rs - r * g.KW;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ih = cih0 + r * g.dh, iw = ciw0 + s * g.dw;
        ra[i] = (cok && k + i < K && (unsigned)ih < (unsigned)g.H && (unsigned)iw < (unsigned)g.W)
                    ? cx[((long long)ih * g.W + iw) * g.Cs + ci]
                    : 0.f;
        if (++s == g.KW) {
          s = 0;
          if (++r == g.KH) {
            r = 0;
            ++ci;
          }
        }
      }
    } else if (!ta) {  // A[m][k]: k contiguous
      const int m = m0 + a_r, k = k0 + a_k;
      const float* src = A + (long long)m * lda + k;
      if (m < M && va && k + 3 < K) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) ra[i] = (m < M && k + i < K) ? src[i] : 0.f;
      }
    } else {  // A[k][m]: m contiguous
      const int m = m0 + a_r, k = k0 + a_k;
      const float* src = A + (long long)k * lda + m;
      if (k < K && va && m + 3 < M) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) ra[i] = (k < K && m + i < M) ? src[i] : 0.f;
      }
    }
    if (!tb) {  // B[k][n]: n contiguous
      const int n = n0 + b_r, k = k0 + b_k;
      const float* src = B + (long long)k * ldb + n;
      if (k < K && vb && n + 3 < N) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) rb[i] = (k < K && n + i < N) ? src[i] : 0.f;
      }
    } else {  // B[n][k]: k contiguous
      const int n = n0 + b_r, k = k0 + b_k;
      const float* src = B + (long long)n * ldb + k;
      if (n < N && vb && k + 3 < K) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) rb[i] = (n < N && k + i < K) ? src[i] : 0.f;
      }
    }
  };
  auto store = [&](int buf) {
    if (!ta) {
#pragma unroll
      for (int i = 0; i < 4; ++i) As[buf][a_k + i][a_r] = ra[i];
    } else {
      *reinterpret_cast<float4*>(&As[buf][a_k][a_r]) = make_float4(ra[0], ra[1], ra[2], ra[3]);
    }
    if (tb) {
#pragma unroll
      for (int i = 0; i < 4; ++i) Bs[buf][b_k + i][b_r] = rb[i];
    } else {
      *reinterpret_cast<float4*>(&Bs[buf][b_k][b_r]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  if (K > 0) {
    load(0);
    store(0);
  }
  __syncthreads();
  for (int k0 = 0, buf = 0; k0 < K; k0 += kSgBK, buf ^= 1) {
    const bool more = k0 + kSgBK < K;
    if (more) load(k0 + kSgBK);
#pragma unroll
    for (int kk = 0; kk < kSgBK; ++kk) {
      float av[8], bv[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + 64]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + 64]);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
      av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
      bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    // the buffer written here was last read in the previous step, before the
    // barrier that ended it; the barrier below publishes it for the next step
    if (more) store(buf ^ 1);
    __syncthreads();
  }
  const bool vy = (ldy & 3) == 0 && aligned16(Y) && (!R || ((ldr & 3) == 0 && aligned16(R)));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + ty * 4 + (i & 3) + (i >> 2) * 64;
    if (gm >= M) continue;
#pragma unroll
    for (int jg = 0; jg < 2; ++jg) {
      const int gn = n0 + tx * 4 + jg * 64;
      if (gn >= N) continue;
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = 0.f;
        if (gn + j < N) {
          v[j] = epi(acc[i][jg * 4 + j], scale, shift, gn + j);
          if (R) v[j] += R[(long long)gm * ldr + gn + j];
          if (relu) v[j] = v[j] > 0.f ? v[j] : 0.f;
        }
      }
      float* dst = Y + (long long)gm * ldy + gn;
      if (vy && gn + 3 < N) {
        *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (gn + j < N) dst[j] = v[j];
      }
    }
  }
}

int gemm_simt_launch(const float* a, const float* b, int batches, const long long* a_off,
                     const long long* b_off, long long y_bstride, int M, int N, int K, int lda,
                     int ldb, int ta, int tb, const float* scale, const float* shift,
                     const float* res, int ldr, int relu, float* y, int ldy, cudaStream_t st) {
  if (M == 0 || N == 0 || batches == 0) return 0;
  dim3 grid((N + kSgBN - 1) / kSgBN, (M + kSgBM - 1) / kSgBM, batches);
  gemm_simt_kernel<false><<<grid, 256, 0, st>>>(a, b, a_off, b_off, y_bstride, M, N, K, lda, ldb, ta,
                                                 tb, scale, shift, res, ldr, relu, y, ldy, SimtConvGeom{});
  return (int)cudaGetLastError();
}

// Ungrouped convolution (NHWC input with channel stride Cs, OIHW weights, output
// [pixel][c_out]) as the implicit GEMM above; the caller keeps N*OH*OW / 128
// within the grid's y limit and C*KH*KW within int.
int conv_simt_igemm_launch(const float* x, int N, int H, int W, int C, int Cs, const float* w, int CO,
                           int KH, int KW, int sh, int sw, int ph, int pw, int dh, int dw, int OH, int OW,
                           const float* scale, const float* shift, const float* res, int relu, float* y,
                           cudaStream_t st) {
  const int M = N * OH * OW, K = C * KH * KW;
  if (M == 0 || CO == 0) return 0;
  const SimtConvGeom g{H, W, Cs, OH, OW, KH, KW, sh, sw, ph, pw, dh, dw};
  dim3 grid((CO + kSgBN - 1) / kSgBN, (M + kSgBM - 1) / kSgBM, 1);
  gemm_simt_kernel<true><<<grid, 256, 0, st>>>(x, w, nullptr, nullptr, 0, M, CO, K, 0, K, 0, 1, scale,
                                                shift, res, CO, relu, y, CO, g);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ weight packing
__global__ void pack_b_kernel(const float* __restrict__ src, int rows, int K, int Kpad, int Cs,
                              int Creal, int rpg, long long gs, long long rs, long long ts,
                              long long cs, int prec, void* hi, void* lo, int pair_kw, int pair_odd) {
  const long long total = (long long)rows * Kpad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / Kpad);
    const int k = (int)(i % Kpad);
    float v = 0.f;
    if (k < K) {
      int tap = k / Cs, c = k % Cs;
      if (pair_kw) {  // pixel pairs: k = (r*KWp + q')*2Cs + h*Cs + c
        const int kwp = (pair_kw + pair_odd + 1) / 2;
        const int tp = k / (2 * Cs), c8 = k - tp * 2 * Cs;
        const int r = tp / kwp, q = 2 * (tp - r * kwp) + c8 / Cs - pair_odd;
        c = c8 % Cs;
        tap = (q >= 0 && q < pair_kw) ? r * pair_kw + q : -1;
      }
      if (tap >= 0 && c < Creal)
        v = src[(long long)(row / rpg) * gs + (long long)(row % rpg) * rs + tap * ts + c * cs];
    }
    if (prec == kPrecBF16) {
      reinterpret_cast<__nv_bfloat16*>(hi)[i] = __float2bfloat16_rn(v);
    } else if (prec == kPrecFP32) {
      reinterpret_cast<float*>(hi)[i] = v;
    } else if (prec == kPrec3xTF32) {
      // hi = the truncated tf32 the tensor core reads from an fp32 container,
      // lo = the remainder rounded to tf32 (the activations are split the same
      // way on the fly)
      const float h = tf32_trunc(v);
      reinterpret_cast<float*>(hi)[i] = h;
      reinterpret_cast<float*>(lo)[i] = to_tf32(v - h);
    } else {
      reinterpret_cast<float*>(hi)[i] = to_tf32(v);
    }
  }
}

int pack_b_launch(const float* src, int rows, int K, int Kpad, int Cs, int Creal, int rpg,
                  long long gs, long long rs, long long ts, long long cs, int prec, void* hi,
                  void* lo, cudaStream_t st, int pair_kw, int pair_odd) {
  const long long total = (long long)rows * Kpad;
  if (total == 0) return 0;
  pack_b_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(src, rows, K, Kpad, Cs, Creal, rpg,
                                                            gs, rs, ts, cs, prec, hi, lo, pair_kw,
                                                            pair_odd);
  return (int)cudaGetLastError();
}

// Two 1x1 convolutions' weights side by side along K, each row scaled by its
// branch's factor; split like pack_b_kernel.
__global__ void pack_dual_b_kernel(const float* __restrict__ w1, const float* __restrict__ s1, int K1,
                                   const float* __restrict__ w2, const float* __restrict__ s2, int K2,
                                   int rows, int prec, void* hi, void* lo) {
  const int Kp = K1 + K2;
  const long long total = (long long)rows * Kp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / Kp);
    const int k = (int)(i % Kp);
    const float v = k < K1 ? w1[(long long)row * K1 + k] * (s1 ? s1[row] : 1.f)
                           : w2[(long long)row * K2 + (k - K1)] * (s2 ? s2[row] : 1.f);
    if (prec == kPrecBF16) {
      reinterpret_cast<__nv_bfloat16*>(hi)[i] = __float2bfloat16_rn(v);
    } else if (prec == kPrec3xTF32) {
      const float h = tf32_trunc(v);
      reinterpret_cast<float*>(hi)[i] = h;
      reinterpret_cast<float*>(lo)[i] = to_tf32(v - h);
    } else {
      reinterpret_cast<float*>(hi)[i] = to_tf32(v);
    }
  }
}

int pack_dual_b_launch(const float* w1, const float* s1, int K1, const float* w2, const float* s2, int K2,
                       int rows, int prec, void* hi, void* lo, cudaStream_t st) {
  const long long total = (long long)rows * (K1 + K2);
  if (total == 0) return 0;
  pack_dual_b_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(w1, s1, K1, w2, s2, K2, rows, prec, hi, lo);
  return (int)cudaGetLastError();
}

__global__ void vec_add_kernel(const float* a, const float* b, float* y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = a[i] + b[i];
}

int vec_add_launch(const float* a, const float* b, float* y, int n, cudaStream_t st) {
  if (n == 0) return 0;
  vec_add_kernel<<<(n + 255) / 256, 256, 0, st>>>(a, b, y, n);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ layout repacks
// 32x32 tiles through shared memory: NCHW [n][c][hw] <-> NHWC [n][hw][c].
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ x, int C, int HW, int Cp,
                                    float* __restrict__ y) {
  __shared__ float t[32][33];
  const int n = blockIdx.z;
  const int hw0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* xn = x + (long long)n * C * HW;
  float* yn = y + (long long)n * HW * Cp;
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int c = c0 + j, hw = hw0 + threadIdx.x;
    t[j][threadIdx.x] = (c < C && hw < HW) ? xn[(long long)c * HW + hw] : 0.f;
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int hw = hw0 + j, c = c0 + threadIdx.x;
    if (hw < HW && c < Cp) yn[(long long)hw * Cp + c] = t[threadIdx.x][j];
  }
}

// Few channels (an RGB image padded to 4 or 8): one thread per pixel, reading
// each plane coalesced along the pixels and writing its padded channel row as
// 16-byte vectors.
template <int CP4>
__global__ void nchw_to_nhwc_small_kernel(const float* __restrict__ x, long long npix, int C,
                                          int HW, float4* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < npix;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / HW;
    const int hw = (int)(i - n * HW);
    const float* px = x + n * C * HW + hw;
    float v[4 * CP4];
#pragma unroll
    for (int c = 0; c < 4 * CP4; ++c) v[c] = c < C ? __ldg(px + (long long)c * HW) : 0.f;
#pragma unroll
    for (int j = 0; j < CP4; ++j)
      y[i * CP4 + j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

int nchw_to_nhwc_launch(const float* x, int N, int C, int H, int W, int Cp, float* y,
                        cudaStream_t st) {
  const int HW = H * W;
  if ((long long)N * HW * Cp == 0) return 0;
  if ((Cp == 4 || Cp == 8) && C <= Cp && ((uintptr_t)y & 15) == 0) {
    const long long npix = (long long)N * HW;
    const int blocks = (int)std::min<long long>((npix + 255) / 256, 148LL * 16);
    if (Cp == 4)
      nchw_to_nhwc_small_kernel<1><<<blocks, 256, 0, st>>>(x, npix, C, HW, (float4*)y);
    else
      nchw_to_nhwc_small_kernel<2><<<blocks, 256, 0, st>>>(x, npix, C, HW, (float4*)y);
    return (int)cudaGetLastError();
  }
  dim3 grid((HW + 31) / 32, (Cp + 31) / 32, N);
  nchw_to_nhwc_kernel<<<grid, dim3(32, 8), 0, st>>>(x, C, HW, Cp, y);
  return (int)cudaGetLastError();
}

__global__ void nhwc_to_nchw_kernel(const float* __restrict__ x, int C, int HW, int Cs,
                                    float* __restrict__ y) {
  __shared__ float t[32][33];
  const int n = blockIdx.z;
  const int hw0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* xn = x + (long long)n * HW * Cs;
  float* yn = y + (long long)n * C * HW;
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int hw = hw0 + j, c = c0 + threadIdx.x;
    t[j][threadIdx.x] = (hw < HW && c < C) ? xn[(long long)hw * Cs + c] : 0.f;
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int c = c0 + j, hw = hw0 + threadIdx.x;
    if (c < C && hw < HW) yn[(long long)c * HW + hw] = t[threadIdx.x][j];
  }
}

int nhwc_to_nchw_launch(const float* x, int N, int C, int H, int W, int Cs, float* y,
                        cudaStream_t st) {
  const int HW = H * W;
  if ((long long)N * HW * C == 0) return 0;
  dim3 grid((HW + 31) / 32, (C + 31) / 32, N);
  nhwc_to_nchw_kernel<<<grid, dim3(32, 8), 0, st>>>(x, C, HW, Cs, y);
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ MaxPool
// max_pool (src/ops/nn/pool.rs:307-393): init f32::MIN, in-bounds taps only,
// fmaxf ignores NaN like f32::max.  Vector path: one thread per (pixel, 4 channels).
__global__ void maxpool_nhwc_v4_kernel(const float* __restrict__ x, int N, int C4, int Cs, int H,
                                       int W, int KH, int KW, int sh, int sw, int pt, int pl,
                                       int OH, int OW, float* __restrict__ y) {
  const long long total = (long long)N * OH * OW * C4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c4 = (int)(i % C4);
    const long long pix = i / C4;
    const int ow = (int)(pix % OW);
    const int oh = (int)((pix / OW) % OH);
    const int n = (int)(pix / ((long long)OW * OH));
    float4 m = make_float4(-3.40282347e+38f, -3.40282347e+38f, -3.40282347e+38f, -3.40282347e+38f);
    for (int r = 0; r < KH; ++r) {
      const int ih = oh * sh - pt + r;
      if ((unsigned)ih >= (unsigned)H) continue;
      for (int s = 0; s < KW; ++s) {
        const int iw = ow * sw - pl + s;
        if ((unsigned)iw >= (unsigned)W) continue;
        const float4 v =
            *reinterpret_cast<const float4*>(x + (((long long)n * H + ih) * W + iw) * Cs + 4 * c4);
        m.x = fmaxf(m.x, v.x);
        m.y = fmaxf(m.y, v.y);
        m.z = fmaxf(m.z, v.z);
        m.w = fmaxf(m.w, v.w);
      }
    }
    *reinterpret_cast<float4*>(y + pix * (long long)Cs + 4 * c4) = m;
  }
}

// 3x3 stride-2 MaxPool (the ResNet stem's) over output-row segments: a thread
// takes P consecutive outputs of one row for 4 channels and loads each input
// vector of the segment's three input rows once (2P+1 per row where per-output
// threads load 3P; longer segments lose more to fewer threads in flight than
// they save in loads).  Per output the maxima are taken in the same order as
// maxpool_nhwc_v4_kernel (rows, then columns), so the results are identical.
template <int P>
__global__ void maxpool3s2_nhwc_v4_kernel(const float4* __restrict__ x, int C4, int Cs4, int H, int W,
                                          int pt, int pl, int OH, int OW, int nseg, unsigned total,
                                          float4* __restrict__ y) {
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int c4 = (int)(i % (unsigned)C4);
    unsigned t = i / (unsigned)C4;
    const int seg = (int)(t % (unsigned)nseg);
    t /= (unsigned)nseg;
    const int oh = (int)(t % (unsigned)OH);
    const unsigned n = t / (unsigned)OH;
    const int ow0 = seg * P, iw0 = 2 * ow0 - pl;
    float4 m[P];
#pragma unroll
    for (int q = 0; q < P; ++q)
      m[q] = make_float4(-3.40282347e+38f, -3.40282347e+38f, -3.40282347e+38f, -3.40282347e+38f);
    for (int r = 0; r < 3; ++r) {
      const int ih = 2 * oh - pt + r;
      if ((unsigned)ih >= (unsigned)H) continue;
      const float4* row = x + ((size_t)n * H + ih) * W * Cs4 + c4;
#pragma unroll
      for (int j = 0; j < 2 * P + 1; ++j) {
        const int iw = iw0 + j;
        if ((unsigned)iw >= (unsigned)W) continue;
        const float4 v = __ldg(row + (size_t)iw * Cs4);
#pragma unroll
        for (int q = 0; q < P; ++q)
          if (j >= 2 * q && j <= 2 * q + 2) {
            m[q].x = fmaxf(m[q].x, v.x);
            m[q].y = fmaxf(m[q].y, v.y);
            m[q].z = fmaxf(m[q].z, v.z);
            m[q].w = fmaxf(m[q].w, v.w);
          }
      }
    }
    float4* yo = y + (((size_t)n * OH + oh) * OW + ow0) * Cs4 + c4;
#pragma unroll
    for (int q = 0; q < P; ++q)
      if (ow0 + q < OW) yo[(size_t)q * Cs4] = m[q];
  }
}

// Scalar path with indices: the ONNX flat NCHW index of the first maximum.
__global__ void maxpool_nhwc_idx_kernel(const float* __restrict__ x, int N, int C, int Cs, int H,
                                        int W, int KH, int KW, int sh, int sw, int pt, int pl,
                                        int OH, int OW, float* __restrict__ y,
                                        long long* __restrict__ ind) {
  const long long total = (long long)N * OH * OW * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long pix = i / C;
    const int ow = (int)(pix % OW);
    const int oh = (int)((pix / OW) % OH);
    const int n = (int)(pix / ((long long)OW * OH));
    float m = -3.40282347e+38f;
    long long mi = -1;
    for (int r = 0; r < KH; ++r) {
      const int ih = oh * sh - pt + r;
      if ((unsigned)ih >= (unsigned)H) continue;
      for (int s = 0; s < KW; ++s) {
        const int iw = ow * sw - pl + s;
        if ((unsigned)iw >= (unsigned)W) continue;
        const float v = x[(((long long)n * H + ih) * W + iw) * Cs + c];
        if (v > m || (mi < 0 && v == m)) {
          m = v;
          mi = (((long long)n * C + c) * H + ih) * W + iw;
        }
      }
    }
    y[pix * Cs + c] = m;
    if (ind) ind[(((long long)n * C + c) * OH + oh) * OW + ow] = mi;
  }
}

int maxpool_nhwc_launch(const float* x, int N, int C, int Cs, int H, int W, int KH, int KW, int sh,
                        int sw, int pt, int pl, int OH, int OW, float* y, long long* ind,
                        cudaStream_t st) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (!ind && C % 4 == 0 && Cs % 4 == 0 && aligned && KH == 3 && KW == 3 && sh == 2 && sw == 2) {
    constexpr int kP = 2;  // outputs per thread (1 / 2 / 4 / 8: 0.236 / 0.224 / 0.303 / 0.525 ms at batch 256)
    const int nseg = (OW + kP - 1) / kP;
    const long long total = (long long)N * OH * nseg * (C / 4);
    if (total == 0) return 0;
    if (total < (1ll << 31)) {
      maxpool3s2_nhwc_v4_kernel<kP><<<grid_for(total, kBlock), kBlock, 0, st>>>(
          reinterpret_cast<const float4*>(x), C / 4, Cs / 4, H, W, pt, pl, OH, OW, nseg, (unsigned)total,
          reinterpret_cast<float4*>(y));
      return (int)cudaGetLastError();
    }
  }
  if (!ind && C % 4 == 0 && Cs % 4 == 0 && aligned) {
    const long long total = (long long)N * OH * OW * (C / 4);
    if (total == 0) return 0;
    maxpool_nhwc_v4_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(
        x, N, C / 4, Cs, H, W, KH, KW, sh, sw, pt, pl, OH, OW, y);
  } else {
    const long long total = (long long)N * OH * OW * C;
    if (total == 0) return 0;
    maxpool_nhwc_idx_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(
        x, N, C, Cs, H, W, KH, KW, sh, sw, pt, pl, OH, OW, y, ind);
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ GlobalAveragePool
// global_pool (src/ops/nn/pool.rs:493-557): each thread sums its channel over
// H*W sequentially in fp32 (the reference's order) and divides by the count.
__global__ void gap_nhwc_kernel(const float* __restrict__ x, int C, int HW,
                                float* __restrict__ y) {
  const int n = blockIdx.y;
  const int c4 = blockIdx.x * blockDim.x + threadIdx.x;
  if (4 * c4 >= C) return;
  const float* p = x + (long long)n * HW * C + 4 * c4;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < HW; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(p + (long long)i * C);
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
  }
  const float cnt = (float)HW;
  *reinterpret_cast<float4*>(y + (long long)n * C + 4 * c4) =
      make_float4(s.x / cnt, s.y / cnt, s.z / cnt, s.w / cnt);
}

__global__ void gap_nhwc_scalar_kernel(const float* __restrict__ x, int C, int HW,
                                       float* __restrict__ y) {
  const int n = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float* p = x + (long long)n * HW * C + c;
  float s = 0.f;
  for (int i = 0; i < HW; ++i) s += p[(long long)i * C];
  y[(long long)n * C + c] = s / (float)HW;
}

// bf16 activations (BF16 precision in a graph): 8 channels (16 bytes) per
// thread, compared / summed in fp32.
__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float (&f)[8]) {
  f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xFFFF0000u);
  f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xFFFF0000u);
  f[4] = __uint_as_float(v.z << 16); f[5] = __uint_as_float(v.z & 0xFFFF0000u);
  f[6] = __uint_as_float(v.w << 16); f[7] = __uint_as_float(v.w & 0xFFFF0000u);
}

__global__ void maxpool_nhwc_bf16_kernel(const uint4* __restrict__ x, int N, int C8, int H, int W, int KH,
                                         int KW, int sh, int sw, int pt, int pl, int OH, int OW,
                                         uint4* __restrict__ y) {
  const long long total = (long long)N * OH * OW * C8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c8 = (int)(i % C8);
    const long long pix = i / C8;
    const int ow = (int)(pix % OW);
    const int oh = (int)((pix / OW) % OH);
    const int n = (int)(pix / ((long long)OW * OH));
    float m[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) m[e] = -3.40282347e+38f;
    for (int r = 0; r < KH; ++r) {
      const int ih = oh * sh - pt + r;
      if ((unsigned)ih >= (unsigned)H) continue;
      for (int q = 0; q < KW; ++q) {
        const int iw = ow * sw - pl + q;
        if ((unsigned)iw >= (unsigned)W) continue;
        float f[8];
        bf16x8_to_f32(x[(((long long)n * H + ih) * W + iw) * C8 + c8], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) m[e] = fmaxf(m[e], f[e]);
      }
    }
    // the maxima are input values, so the conversion back is exact
    uint4 o;
    o.x = (__float_as_uint(m[1]) & 0xFFFF0000u) | (__float_as_uint(m[0]) >> 16);
    o.y = (__float_as_uint(m[3]) & 0xFFFF0000u) | (__float_as_uint(m[2]) >> 16);
    o.z = (__float_as_uint(m[5]) & 0xFFFF0000u) | (__float_as_uint(m[4]) >> 16);
    o.w = (__float_as_uint(m[7]) & 0xFFFF0000u) | (__float_as_uint(m[6]) >> 16);
    y[pix * C8 + c8] = o;
  }
}

int maxpool_nhwc_bf16_launch(const void* x, int N, int C, int H, int W, int KH, int KW, int sh, int sw,
                             int pt, int pl, int OH, int OW, void* y, cudaStream_t st) {
  if (C % 8 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15))
    return (int)cudaErrorMisalignedAddress;
  const long long total = (long long)N * OH * OW * (C / 8);
  if (total == 0) return 0;
  maxpool_nhwc_bf16_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(
      static_cast<const uint4*>(x), N, C / 8, H, W, KH, KW, sh, sw, pt, pl, OH, OW, static_cast<uint4*>(y));
  return (int)cudaGetLastError();
}

__global__ void gap_nhwc_bf16_kernel(const uint4* __restrict__ x, int C8, int HW, float* __restrict__ y) {
  const int n = blockIdx.y;
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 >= C8) return;
  const uint4* p = x + (long long)n * HW * C8 + c8;
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < HW; ++i) {
    float f[8];
    bf16x8_to_f32(p[(long long)i * C8], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] += f[e];
  }
  const float cnt = (float)HW;
  float4* o = reinterpret_cast<float4*>(y + (long long)n * C8 * 8 + 8 * c8);
  o[0] = make_float4(s[0] / cnt, s[1] / cnt, s[2] / cnt, s[3] / cnt);
  o[1] = make_float4(s[4] / cnt, s[5] / cnt, s[6] / cnt, s[7] / cnt);
}

int gap_nhwc_bf16_launch(const void* x, int N, int C, int HW, float* y, cudaStream_t st) {
  if (N == 0 || C == 0) return 0;
  if (C % 8 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15))
    return (int)cudaErrorMisalignedAddress;
  const int c8 = C / 8;
  const int block = c8 < 128 ? 32 * ((c8 + 31) / 32) : 128;
  dim3 grid((c8 + block - 1) / block, N);
  gap_nhwc_bf16_kernel<<<grid, block, 0, st>>>(static_cast<const uint4*>(x), c8, HW, y);
  return (int)cudaGetLastError();
}

int gap_nhwc_launch(const float* x, int N, int C, int HW, float* y, cudaStream_t st) {
  if (N == 0 || C == 0) return 0;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (C % 4 == 0 && aligned) {
    const int c4 = C / 4;
    const int block = c4 < 128 ? 32 * ((c4 + 31) / 32) : 128;
    dim3 grid((c4 + block - 1) / block, N);
    gap_nhwc_kernel<<<grid, block, 0, st>>>(x, C, HW, y);
  } else {
    dim3 grid((C + 127) / 128, N);
    gap_nhwc_scalar_kernel<<<grid, 128, 0, st>>>(x, C, HW, y);
  }
  return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ elementwise
struct BcastArgs {
  long long shape[8];
  long long as[8];
  long long bs[8];
};

// element_wise_binary_op(+) (src/ops/tensor.rs:1124-1218) without materialising
// the broadcast copies: stride 0 on broadcast dims.
__global__ void add_bcast_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                 float* __restrict__ y, int rank, BcastArgs g, long long total,
                                 int relu) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long rem = i, ia = 0, ib = 0;
    for (int d = rank - 1; d >= 0; --d) {
      const long long c = rem % g.shape[d];
      rem /= g.shape[d];
      ia += c * g.as[d];
      ib += c * g.bs[d];
    }
    float v = a[ia] + b[ib];
    if (relu) v = v > 0.f ? v : 0.f;
    y[i] = v;
  }
}

__global__ void add_same_v4_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                   float4* __restrict__ y, long long n4, int relu) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 u = a[i], v = b[i];
    float4 r = make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w);
    if (relu) {
      r.x = r.x > 0.f ? r.x : 0.f;
      r.y = r.y > 0.f ? r.y : 0.f;
      r.z = r.z > 0.f ? r.z : 0.f;
      r.w = r.w > 0.f ? r.w : 0.f;
    }
    y[i] = r;
  }
}

int add_broadcast_launch(const float* a, const float* b, float* y, int rank,
                         const long long* shape, const long long* as, const long long* bs,
                         long long total, int relu, cudaStream_t st) {
  if (total == 0) return 0;
  bool same = true;
  long long expect = 1;
  for (int d = rank - 1; d >= 0; --d) {
    if (shape[d] != 1 && (as[d] != expect || bs[d] != expect)) same = false;
    expect *= shape[d];
  }
  const bool aligned = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (same && total % 4 == 0 && aligned) {
    add_same_v4_kernel<<<grid_for(total / 4, kBlock), kBlock, 0, st>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
        reinterpret_cast<float4*>(y), total / 4, relu);
  } else {
    BcastArgs g{};
    for (int d = 0; d < rank; ++d) {
      g.shape[d] = shape[d];
      g.as[d] = as[d];
      g.bs[d] = bs[d];
    }
    add_bcast_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(a, b, y, rank, g, total, relu);
  }
  return (int)cudaGetLastError();
}

// 3-D convolution, NCDHW in and out, weights [CO][C/group][KD][KH][KW]: one
// thread per output element, fp32 fused multiply-adds over (ci, kd, kh, kw) in
// that order, taps outside the input skipped (zero padding).  The reference's
// compute_conv3d_direct_impl (src/ops/nn/conv.rs:937-1038) as a CUDA-core
// kernel; consecutive threads take consecutive output columns.
__global__ void conv3d_direct_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                     const float* __restrict__ bias, float* __restrict__ y, Conv3dArgs a) {
  const long long total = (long long)a.N * a.CO * a.OD * a.OH * a.OW;
  const int cg = a.C / a.G, cog = a.CO / a.G;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i;
    const int ow = (int)(r % a.OW); r /= a.OW;
    const int oh = (int)(r % a.OH); r /= a.OH;
    const int od = (int)(r % a.OD); r /= a.OD;
    const int co = (int)(r % a.CO);
    const int n = (int)(r / a.CO);
    const int g = co / cog;
    float acc = 0.f;
    const float* wc = w + (long long)co * cg * a.KD * a.KH * a.KW;
    for (int ci = 0; ci < cg; ++ci) {
      const float* xc = x + ((long long)n * a.C + (long long)g * cg + ci) * a.D * a.H * a.W;
      for (int kd = 0; kd < a.KD; ++kd) {
        const int id = od * a.sd - a.pd + kd * a.dd;
        if ((unsigned)id >= (unsigned)a.D) continue;
        for (int kh = 0; kh < a.KH; ++kh) {
          const int ih = oh * a.sh - a.ph + kh * a.dh;
          if ((unsigned)ih >= (unsigned)a.H) continue;
          const float* xr = xc + ((long long)id * a.H + ih) * a.W;
          const float* wr = wc + ((long long)(ci * a.KD + kd) * a.KH + kh) * a.KW;
          for (int kw = 0; kw < a.KW; ++kw) {
            const int iw = ow * a.sw - a.pw + kw * a.dw;
            if ((unsigned)iw < (unsigned)a.W) acc = fmaf(xr[iw], wr[kw], acc);
          }
        }
      }
    }
    if (bias) acc += bias[co];
    if (a.relu) acc = acc > 0.f ? acc : 0.f;
    y[i] = acc;
  }
}

int conv3d_direct_launch(const float* x, const float* w, const float* bias, float* y, const Conv3dArgs& a,
                         cudaStream_t st) {
  const long long total = (long long)a.N * a.CO * a.OD * a.OH * a.OW;
  if (total == 0) return 0;
  conv3d_direct_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(x, w, bias, y, a);
  return (int)cudaGetLastError();
}

// relu (src/ops/activations.rs:244-246): v > 0 ? v : 0 (NaN -> 0).
__device__ __forceinline__ float relu1(float v) { return v > 0.f ? v : 0.f; }

__global__ void relu_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = relu1(x[i]);
}

// 16-byte vectors over the first n & ~3 elements (both pointers 16-byte aligned);
// the first threads of block 0 take the last n & 3.
__global__ void relu_v4_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  const long long n4 = n >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4* y4 = reinterpret_cast<float4*>(y);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 v = x4[i];
    y4[i] = make_float4(relu1(v.x), relu1(v.y), relu1(v.z), relu1(v.w));
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const long long i = (n4 << 2) + threadIdx.x;
    y[i] = relu1(x[i]);
  }
}

int relu_launch(const float* x, float* y, long long n, cudaStream_t st) {
  if (n == 0) return 0;
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0)
    relu_v4_kernel<<<grid_for(n >> 2, kBlock), kBlock, 0, st>>>(x, y, n);
  else
    relu_kernel<<<grid_for(n, kBlock), kBlock, 0, st>>>(x, y, n);
  return (int)cudaGetLastError();
}

// y = x * scale[c] + shift[c] over [outer][C][inner] (NCHW: inner = H*W;
// NHWC: outer = N*H*W, inner = 1).
__global__ void channel_affine_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                      const float* __restrict__ shift, float* __restrict__ y,
                                      long long outer, int C, long long inner, int relu) {
  const long long total = outer * C * inner;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)((i / inner) % C);
    float v = x[i] * scale[c] + shift[c];
    if (relu) v = v > 0.f ? v : 0.f;
    y[i] = v;
  }
}

int channel_affine_launch(const float* x, const float* scale, const float* shift, float* y,
                          long long outer, int C, long long inner, int relu, cudaStream_t st) {
  const long long total = outer * C * inner;
  if (total == 0) return 0;
  channel_affine_kernel<<<grid_for(total, kBlock), kBlock, 0, st>>>(x, scale, shift, y, outer, C,
                                                                    inner, relu);
  return (int)cudaGetLastError();
}

// BatchNormalization folded to a per-channel affine of the conv accumulator.
__global__ void bn_fold_kernel(const float* gamma, const float* beta, const float* mean,
                               const float* var, const float* bias, float eps, int C,
                               float* scale, float* shift) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float s = gamma[c] / sqrtf(var[c] + eps);
  const float b = bias ? bias[c] : 0.f;
  scale[c] = s;
  shift[c] = beta[c] + (b - mean[c]) * s;
}

int bn_fold_launch(const float* gamma, const float* beta, const float* mean, const float* var,
                   const float* bias, float eps, int C, float* scale, float* shift,
                   cudaStream_t st) {
  if (C == 0) return 0;
  bn_fold_kernel<<<(C + 127) / 128, 128, 0, st>>>(gamma, beta, mean, var, bias, eps, C, scale,
                                                  shift);
  return (int)cudaGetLastError();
}

}  // namespace ob2
