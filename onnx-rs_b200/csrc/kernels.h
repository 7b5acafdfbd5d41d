// Device-kernel launch interface shared by the C-ABI layer and the kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ob2 {

enum Precision { kPrec3xTF32 = 0, kPrecTF32 = 1, kPrecBF16 = 2, kPrecFP32 = 3 };

// Implicit-GEMM problem: D[b][m][n] = sum_k A_b[m][k] * B_b[n][k], then the
// epilogue  y = D * scale[n] + shift[n] (+ residual) (relu).
//   A rows are output pixels of a convolution over an NHWC input (a plain
//   row-major matrix is the 1x1 / stride-1 / H=1 special case); K is ordered
//   (kh, kw, c) with c fastest, c padded to `Cs` channels per pixel.
//   B is the packed weight matrix [rows][Kpad] (K-major), read through TMA.
struct IgemmParams {
  const float* x;      // NHWC activations (or row-major A)
  int Hin, Win, Cs;    // input height, width, channels per pixel (multiple of 4)
  int OH, OW;          // output height, width
  int KW;              // filter width
  int sh, sw, ph, pw, dh, dw;
  int M;               // rows per batch = N*OH*OW (or matrix M)
  int Nc;              // columns (output channels / matrix N), multiple of 4
  int K;               // KH*KW*Cs (real K)
  int num_kb;          // ceil(K / 32)
  int batches;         // independent GEMMs (MatMul batch); 1 for conv
  const long long* a_off;  // per-batch element offset into x (nullptr = 0)
  const int* b_row;        // per-batch row offset into B (nullptr = 0)
  long long y_bstride;     // per-batch element stride of y / residual
  float* y;
  int ldy;                 // row stride of y in elements
  const float* scale;      // per-column multiplier (nullptr = 1)
  const float* shift;      // per-column addend (nullptr = 0)
  const float* res;        // residual, same layout as y (nullptr = none)
  int ldr;
  int relu;
  int* status;             // device status word (ONNXB200_ERR_* on failure)
  int m_tiles, n_tiles;
  // How A tiles reach shared memory: kALoadGather = per-thread 16-byte copies
  // (any shape), kALoadTma2d = TMA tile of the [rows][Cs] matrix (1x1 stride-1
  // convs, GEMMs; Cs >= 32), kALoadIm2col = TMA im2col over the NHWC tensor, 32
  // channels of one filter tap per k-block (Cs % 32 == 0), kALoadIm2colTaps =
  // TMA im2col of 32 / Cs whole filter taps per k-block (Cs = 4, 8 or 16, e.g.
  // an RGB stem).
  int a_mode;
  // Second A source (0 = none): k-blocks kb >= kb_split read a 1x1, pad-0
  // convolution of stride s2 over another NHWC tensor x2 ([N][H2][W2][Cs2])
  // at the same output pixels, so that two convolutions whose outputs are
  // added (a bottleneck's last 1x1 and its projection shortcut) share one
  // K loop and one accumulator; B holds both weight matrices back to back
  // along K.  Source 1 is then a kALoadTma2d problem with K1 = kb_split * 32.
  int kb_split;
  const float* x2;
  int H2, W2, Cs2, s2;
  int a_mode2;             // kALoadTma2d (stride 1) or kALoadIm2col
  // BF16 precision only: the activations (x, x2) are stored as bf16 (k-blocks of
  // 64 elements, Cs a multiple of 64, TMA modes only), and / or the output y and
  // the residual are stored as bf16.  x / y / res then point at bf16 data.
  int a_bf16;
  int out_bf16;
  // K split (0 or 1 = none): see igemm_launch_split.  Inside the kernel the
  // problem is then `ksplit` batches over the same A and B (batches == ksplit),
  // batch b running k-blocks [b * num_kb / ksplit, (b + 1) * num_kb / ksplit).
  int ksplit;
  // Output rows of A (pixels) before this problem's row 0: a problem that is the
  // tail of a larger one reads A (and computes pixel coordinates) at rows
  // m_base + m, while y, the residual and M stay relative to the tail.
  int m_base;
};

enum ALoadMode { kALoadGather = 0, kALoadTma2d = 1, kALoadIm2col = 2, kALoadIm2colTaps = 3 };

// Encodes the TMA map of the A operand for p.a_mode (x, shape and conv geometry
// from p); returns a CUresult (0 = success).  Not needed for kALoadGather.
int encode_a_map(const IgemmParams& p, int N, CUtensorMap* map);

// Chooses the A load mode for a problem (conv geometry in p; batched GEMMs with
// per-batch A offsets use kALoadTma2d over all rows).
int pick_a_mode(const IgemmParams& p, int precision);

// Picks BN (64/128/256) for a problem; returned value is what launch uses.
int igemm_pick_bn(const IgemmParams& p, int precision, int num_sms);

// The view of the second A source of a two-source problem as a single-source
// problem (x2 and its geometry), for encode_a_map.
IgemmParams second_source_view(const IgemmParams& p);

// Launches the tcgen05 kernel.  tm_hi / tm_lo are TMA maps over the packed
// weights (tm_lo is only read in 3xTF32 mode); tm_a2 is the map of the second
// A source (ignored unless p.kb_split > 0).  Returns a cudaError_t.
int igemm_launch(const IgemmParams& p, const CUtensorMap& tm_hi, const CUtensorMap& tm_lo,
                 const CUtensorMap& tm_a, const CUtensorMap& tm_a2, int precision, int bn, int num_sms,
                 cudaStream_t stream);

// The tcgen05 kernel (3xTF32 / TF32 / BF16 operands from fp32 activations,
// k-blocks of 32) behind igemm_launch.
int igemm3_launch(const IgemmParams& p, const CUtensorMap& tm_hi, const CUtensorMap& tm_lo,
                  const CUtensorMap& tm_a, const CUtensorMap& tm_a2, int precision, int bn, int num_sms,
                  cudaStream_t stream);

// K split: runs the K loop as `ksplit` slices of whole k-blocks (output tiles x
// slices CTAs' worth of work, for problems with too few tiles to fill the GPU),
// each slice storing raw fp32 partial sums to ws ([ksplit][M][Nc], 16-byte
// aligned), then one reduction pass sums the slices in order and applies p's
// epilogue (scale, shift, residual, Relu) into p.y.  ksplit <= 1 is a plain
// igemm_launch.  Single-batch problems with fp32 activations and outputs only.
// split_mt > 0 splits only the tail: M-tiles [0, split_mt) run unsplit first (the
// whole waves of tiles), then rows [split_mt * 128, M) run split, ws holding
// [ksplit][M - split_mt * 128][Nc].
int igemm_launch_split(const IgemmParams& p, int ksplit, int split_mt, float* ws, const CUtensorMap& tm_hi,
                       const CUtensorMap& tm_lo, const CUtensorMap& tm_a, const CUtensorMap& tm_a2,
                       int precision, int bn, int num_sms, cudaStream_t stream);

// Tile width and K split for a problem (geometry in p; `residual`: the epilogue
// adds a residual): igemm_pick_bn's width, or (when a K split is modelled to be
// >= 6% faster: few output tiles or a partial last wave, long K) the split and the width to use with
// it.  *ksplit = 1 means no split.  Only fp32 activations and outputs split.
// *split_mt: the first split M-tile (0 = the whole problem; > 0: only the tail
// past the whole waves of tiles).
void igemm_pick_split(const IgemmParams& p, bool residual, int precision, int num_sms, int* bn, int* ksplit,
                      int* split_mt);

// Sums ksplit slices of [M][N] fp32 partial sums (slice order) and applies the
// epilogue: y = relu(sum * scale + shift + res), all fp32.
int splitk_reduce_launch(const float* ws, int ksplit, int M, int N, float* y, int ldy, const float* scale,
                         const float* shift, const float* res, int ldr, int relu, cudaStream_t stream);

// K elements per k-block of the kernel used for a precision (p.num_kb = Kpad / this):
// 32, or 64 when the activations are stored as bf16 (128-byte rows either way).
inline int igemm_block_k(int, bool a_bf16 = false) { return a_bf16 ? 64 : 32; }
// Padded K (row length of the packed weights): a whole number of k-blocks.
inline int igemm_kpad(long long K, int precision, bool a_bf16 = false) {
  const int bk = igemm_block_k(precision, a_bf16);
  return (int)((K + bk - 1) / bk * bk);
}

// ----------------------------------------------------------------- SIMT kernels
// Direct convolution on CUDA cores (fp32 FFMA), any groups / channel count.
// NHWC in, NHWC out, weights OIHW (original layout), same epilogue.
int conv_direct_launch(const float* x, int N, int H, int W, int C, int Cs, const float* w,
                       int CO, int KH, int KW, int sh, int sw, int ph, int pw, int dh, int dw, int group,
                       int OH, int OW, const float* scale, const float* shift, const float* res,
                       int relu, float* y, cudaStream_t stream);

// Plain batched GEMM on CUDA cores for shapes the tcgen05 kernel does not take.
// C[b] = alpha * op(A[b]) * op(B[b]) ; epilogue as above.
int gemm_simt_launch(const float* a, const float* b, int batches, const long long* a_off,
                     const long long* b_off, long long y_bstride, int M, int N, int K, int lda,
                     int ldb, int trans_a, int trans_b, const float* scale, const float* shift,
                     const float* res, int ldr, int relu, float* y, int ldy, cudaStream_t stream);

// Packs fp32 weights into the K-major [rows][Kpad] operand of the tcgen05
// kernel.  src element (row, k) is read from
//   src[(row/rpg)*gs + (row%rpg)*rs + (k/Cs)*ts + (k%Cs)*cs]
// for k%Cs < Creal, zero otherwise (and zero for k >= K).  For 3xTF32 both hi
// and lo are written; for TF32 only hi; for BF16 `hi` receives bf16 values.
//
// pair_kw > 0 selects the pixel-pair layout of a stride-2 convolution over a
// Cs-channel input read as 2*Cs-channel pixel pairs: k = (r*KWp + q')*2Cs + h*Cs + c
// holds original tap (r, q = 2q' + h - pair_odd) (zero if q is outside [0, pair_kw)),
// with KWp = (pair_kw + pair_odd + 1) / 2; Cs is then the original channel stride.
int pack_b_launch(const float* src, int rows, int K, int Kpad, int Cs, int Creal, int rpg,
                  long long gs, long long rs, long long ts, long long cs, int precision,
                  void* hi, void* lo, cudaStream_t stream, int pair_kw = 0, int pair_odd = 0);

// Packs two 1x1 convolutions' weights ([rows][K1] and [rows][K2], row-major)
// side by side along K, each row scaled by its branch's per-row factor (the
// folded BatchNormalization scale; null = 1): the B operand of a two-source
// problem.  Kpad = K1 + K2 (both multiples of 32).  hi / lo as pack_b_launch.
int pack_dual_b_launch(const float* w1, const float* scale1, int K1, const float* w2, const float* scale2,
                       int K2, int rows, int precision, void* hi, void* lo, cudaStream_t stream);

// y[i] = a[i] + b[i] (n floats; the two branches' folded shifts).
int vec_add_launch(const float* a, const float* b, float* y, int n, cudaStream_t stream);

// NCHW -> NHWC with channel padding to Cp (zero-filled), and NHWC -> NCHW.
int nchw_to_nhwc_launch(const float* x, int N, int C, int H, int W, int Cp, float* y,
                        cudaStream_t stream);
int nhwc_to_nchw_launch(const float* x, int N, int C, int H, int W, int Cs, float* y,
                        cudaStream_t stream);

// MaxPool 2-D over NHWC (channel stride Cs), optional int64 NCHW flat indices.
int maxpool_nhwc_launch(const float* x, int N, int C, int Cs, int H, int W, int KH, int KW,
                        int sh, int sw, int pt, int pl, int OH, int OW, float* y,
                        long long* indices, cudaStream_t stream);

// MaxPool over bf16 NHWC (channels packed, C % 8 == 0), bf16 out.
int maxpool_nhwc_bf16_launch(const void* x, int N, int C, int H, int W, int KH, int KW, int sh, int sw,
                             int pt, int pl, int OH, int OW, void* y, cudaStream_t stream);
// Global average pool of bf16 NHWC (C % 8 == 0) into fp32 y[n][c].
int gap_nhwc_bf16_launch(const void* x, int N, int C, int HW, float* y, cudaStream_t stream);

// Global average pool over NHWC: y[n][c] = mean over H*W.
int gap_nhwc_launch(const float* x, int N, int C, int HW, float* y, cudaStream_t stream);

// Broadcast binary add (rank <= 8) with optional relu; and relu alone.
int add_broadcast_launch(const float* a, const float* b, float* y, int rank,
                         const long long* out_shape, const long long* a_strides,
                         const long long* b_strides, long long total, int relu,
                         cudaStream_t stream);
int relu_launch(const float* x, float* y, long long n, cudaStream_t stream);

// 3-D direct convolution (NCDHW, fp32 on CUDA cores).
struct Conv3dArgs {
  int N, C, D, H, W, CO, G;
  int KD, KH, KW, OD, OH, OW;
  int sd, sh, sw, pd, ph, pw, dd, dh, dw;
  int relu;
};
int conv3d_direct_launch(const float* x, const float* w, const float* bias, float* y, const Conv3dArgs& a,
                         cudaStream_t stream);

// Per-channel affine (BatchNormalization as scale/shift) over NHWC or NCHW.
int channel_affine_launch(const float* x, const float* scale, const float* shift, float* y,
                          long long outer, int C, long long inner, int relu,
                          cudaStream_t stream);

// Computes scale = gamma / sqrt(var + eps), shift = beta + (bias - mean) * scale
// (bias may be null) on the device.
int bn_fold_launch(const float* gamma, const float* beta, const float* mean, const float* var,
                   const float* bias, float eps, int C, float* scale, float* shift,
                   cudaStream_t stream);

}  // namespace ob2
