// tcgen05 implicit-GEMM kernel (3xTF32, TF32 and BF16 modes; fp32 activations
// and outputs): convolution without an im2col buffer, and batched broadcast GEMM.
//
// Replaces the reference's compute_conv2d_im2col + im2col_2d
// (src/ops/nn/conv.rs:1142-1368), the direct 1x1 path (conv.rs:849-935),
// compute_matmul's per-batch sgemm (src/ops/math/matmul.rs:124-279) and
// compute_gemm (src/ops/math/gemm.rs:172-291).
//
// Persistent, warp-specialised, one 416-thread CTA per SM.  Tile 128 x BN
// (BN = 64 or 128; 256 in TF32), k-blocks of 32 fp32 (128-byte swizzled rows:
// TMA moves about one box row per two cycles, so wide rows are fast).
//   warps 0-3   epilogue: TMEM -> registers, per-channel scale/shift (bias, folded
//               BatchNormalization, staged per tile in shared memory), residual,
//               Relu.  Warp w stores (and loads the residual of) its own 32 rows of
//               each 16- or 32-column group with its own TMA boxes (the hardware
//               clips rows >= M and columns >= N).
//   warps 4-7   loaders.  TMA modes: lane 0 of each warp takes every fourth
//               k-block (a TMA issue holds its thread for hundreds of cycles) and
//               issues its A tile (2-D tile of the [pixels][channels] matrix for 1x1
//               stride-1 convs and GEMMs, or an im2col box for k x k convs: the
//               hardware walks 128 output pixels across rows and images, zero fill =
//               padding) and its weight tiles, coordinates worked out before the
//               wait for the stage.  Taps mode (4, 8 or 16 channels): one im2col box per filter
//               tap.  Gather mode (other channel counts): 16-byte cp.async copies
//               with zero fill.
//   warps 8-11  converters: warp 8+q owns TMEM lanes 32q..32q+31 (= tile rows).
//               3xTF32: each thread writes hi = trunc_tf32(v) and lo = rna_tf32(v - hi)
//               of its row to a TMEM A slot; BF16: bf16 pairs; TF32: the MMAs read
//               the raw fp32 A from shared memory (the tensor core uses its upper 19
//               bits), which is only rewritten for taps-mode boxes or K padding.
//   warp 12     TMEM allocation and one thread issuing tcgen05.mma (kind::tf32 or
//               kind::f16), A from TMEM (from shared memory in TF32), B from shared
//               memory.
// The K loop is bound by the number of operand stages in flight: a stage's round
// trip (release -> TMA issue -> landing -> conversion -> MMAs -> commit) takes
// ~5k cycles, of which the TMA issue is ~2k.
// 3xTF32: a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi (Ootomo & Yokota, 2022), with the
// same split for both operands.  With BN = 64 the B hi and lo rows are stacked so
// that one N = 128 MMA computes two of the three products.  The tensor core adds
// into its fp32 accumulator with truncation, so each TMEM accumulator sums only 4
// k-blocks (48 MMAs) and the epilogue warps fold these chunks into a running total
// with round-to-nearest fp32 adds.
//
// Every wait is bounded (kWaitTimeoutNs); on expiry the kernel records
// ONNXB200_ERR_TIMEOUT in the status word and winds down.  The epilogue warps
// take every abort decision together (barrier AND-reduction once per chunk and
// per tile), so none of them is ever left waiting at a named barrier.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace ob2 {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;  // fp32 K elements per k-block: 128-byte rows (TMA moves
                         // about one row per two cycles, so wider rows are faster)
constexpr int kEpiThreads = 128;
constexpr int kLoadWarp0 = 4, kConvWarp0 = 8, kMmaWarp = 12;
constexpr int kThreads = 13 * 32;
constexpr int kSmemBudget = 224 * 1024;
// The epilogue works in groups of EG output columns (a 128 x EG fp32 staging
// tile per TMA store or residual load): EG = 32 (128-byte rows) stores fastest;
// EG = 16 halves the staging memory so that 3xTF32 with BN = 128 fits four 48 KB
// operand stages, which pays when the tile's K loop is long.

// AIO (BF16 only): bit 0 = the activations A are stored as bf16 (read by the
// MMAs straight from shared memory, 64-element k-blocks of 128-byte rows);
// bit 1 = the output and residual are stored as bf16.
template <int PREC, int BN, int EG, int NB, int AIO = 0>
struct Layout {
  static constexpr bool kABf16 = (AIO & 1) != 0;
  static constexpr bool kOBf16 = (AIO & 2) != 0;
  static constexpr int kBK = kABf16 ? 64 : 32;  // K elements per k-block (128-byte A rows)
  static constexpr int kOes = kOBf16 ? 2 : 4;   // bytes per output element
  static constexpr int kEpiTile = kBM * EG * kOes;
  static constexpr int kEpiRow = EG * kOes;     // bytes per staging row (64 or 128)
  static constexpr bool kSplit = (PREC == kPrec3xTF32);
  static constexpr bool kBf16 = (PREC == kPrecBF16);
  static constexpr bool kTmemA = kSplit || (kBf16 && !kABf16);  // converters write A to TMEM
  static constexpr int kARaw = kBM * kBK * (kABf16 ? 2 : 4);   // 16 KB
  static constexpr int kBBytes = BN * kBK * (kBf16 ? 2 : 4);  // one B operand (hi or lo)
  static constexpr int kStage = kARaw + (kSplit ? 2 : 1) * kBBytes;
  static constexpr int kEpiBytes = 2 * NB * kEpiTile;  // out[NB] + res[NB]
  // (256-column tiles also leave room for their 2 KB of staged scale / shift)
  static constexpr int kS1raw = (kSmemBudget - kEpiBytes - (BN > 128 ? 2 * BN * 4 : 0)) / kStage;
  static constexpr int kS1cap = kS1raw > 8 ? 8 : kS1raw;
  static constexpr bool kPromote = kSplit;
  // k-blocks per TMEM accumulator chunk.  With BN = 64 (stacked B, below) the
  // big-term half of the chunk takes only the a_hi.b_hi products: 8 k-blocks give
  // it 32 truncating adds, fewer than the 48 of a 4-k-block three-product chunk.
  static constexpr int kChunkKB = kPromote ? (BN == 64 ? 8 : 4) : (1 << 30);
  // 3xTF32 with BN = 64: B hi and B lo sit back to back in each stage, so one
  // N = 128 MMA computes [a_hi.b_hi | a_hi.b_lo] and an N = 64 MMA adds a_lo.b_hi
  // to the second half: two MMA instructions per K step instead of three (the
  // MMA issue rate of one thread bounds the kernel).  Chunk accumulators are
  // then 128 columns wide (big | small terms), 128-column aligned.
  static constexpr bool kStack = kSplit && BN == 64;
  static constexpr int kChunkCols = kStack ? 128 : BN;
  static constexpr int kAccCols = kPromote ? (kStack ? 384 : 3 * BN) : 2 * BN;
  // 3xTF32: every MMA reads A from TMEM (a slot = hi[32] | lo[32] columns), so
  // shared memory serves only the B operands to the tensor core -- the kernel is
  // bound by shared-memory bandwidth (128 B/cycle/SM), which the A reads of
  // A-from-shared-memory MMAs would take.  The TMEM slots form their own ring
  // (S2 <= S1), reused once the commit of the slot's previous item has fired.
  // TF32: A is read from shared memory as it landed; S2 == S1, no TMEM slots.
  // BF16: A converted to bf16 pairs in TMEM (16 columns per k-block).
  static constexpr int kAStageCols = kSplit ? 2 * kBK : (kBf16 ? kBK / 2 : 0);
  static constexpr int kS2raw = kTmemA ? (512 - kAccCols) / kAStageCols : 64;
  static constexpr int kS1 = kS1cap;
  static constexpr int kS2 = (kTmemA && kS2raw < kS1) ? kS2raw : kS1;
  static_assert(kS2 >= 2, "TMEM too small for two A slots");
  static_assert(kS1 >= 2, "shared memory too small");
  static constexpr int kACol0 = kAccCols;
  static constexpr int kTmemCols = 512;
  static constexpr int kOffOut = 0;                     // out[NB]  (1024-aligned tiles)
  static constexpr int kOffRes = NB * kEpiTile;         // res[NB]
  static constexpr int kOffA = 2 * NB * kEpiTile;       // raw A stages
  static constexpr int kOffB = kOffA + kS1 * kARaw;     // B hi stages
  static constexpr int kBStride = (kStack ? 2 : 1) * kBBytes;  // stage s at kOffB + s * kBStride
  static constexpr int kOffBlo = kStack ? kOffB + kBBytes : kOffB + kS1 * kBBytes;  // B lo stages
  static constexpr int kOffBar = kOffB + kS1 * kBBytes + (kSplit ? kS1 * kBBytes : 0);
  // s1_full[S1], s1_empty[S1], t_full[S2], acc_full[2], acc_empty[2],
  // res_full[4 warps][2], drain
  static constexpr int kNumBars = 2 * kS1 + kS2 + 4 * NB + 7;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kOffSS = (kOffMisc + 16 + 127) / 128 * 128;  // scale[BN], shift[BN]
  static_assert(kOffSS % 16 == 0, "float4 reads of the staged scale / shift");
  static constexpr int kBytes = kOffSS + 2 * BN * 4 + 1024;
  static_assert(kBytes <= 227 * 1024, "exceeds the 227 KB of shared memory per block");
};

// 64-byte-swizzle layout of a [rows][16 fp32] tile: 16-byte chunk c of row r.
__device__ __forceinline__ uint32_t swz64(int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); }
// K-major operand, 64-byte swizzle (bf16 B tiles): 8-row atoms of 512 bytes.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;  // SWIZZLE_64B
  return d;
}
// 128-byte-swizzle layout of a [rows][32 fp32] tile.
__device__ __forceinline__ uint32_t swz128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }
// Staging tile of the epilogue: rows of RB bytes (64 or 128), 16-byte chunk c,
// swizzled like its TMA box.
template <int RB>
__device__ __forceinline__ uint32_t swz_eg(int r, int c) {
  return RB == 128 ? swz128(r, c) : swz64(r, c);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h2);
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ void sts_u4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld_32x32b_x16(taddr, r); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[32]) { tmem_ld_32x32b_x32(taddr, r); }

__device__ __forceinline__ void sts_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

template <int PREC, int BN, int EG, int NB, int AIO>
__global__ void __launch_bounds__(kThreads, 1)
    igemm_tc3_kernel(const __grid_constant__ IgemmParams p, const __grid_constant__ CUtensorMap tm_hi,
                     const __grid_constant__ CUtensorMap tm_lo, const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_a2, const __grid_constant__ CUtensorMap tm_y,
                     const __grid_constant__ CUtensorMap tm_res) {
  using L = Layout<PREC, BN, EG, NB, AIO>;
  constexpr int kBK = L::kBK;
  constexpr int kEG = EG;
  constexpr int kEpiTile = L::kEpiTile;
  constexpr int S1 = L::kS1;
  constexpr int S2 = L::kS2;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_addr);
  const uint32_t out_st = base + L::kOffOut, res_st = base + L::kOffRes;
  const uint32_t a_raw = base + L::kOffA, b_hi = base + L::kOffB, b_lo = base + L::kOffBlo;
  const uint32_t bar0 = base + L::kOffBar;
  auto s1_full = [&](int s) { return bar0 + 8u * s; };
  auto s1_empty = [&](int s) { return bar0 + 8u * (S1 + s); };
  auto t_full = [&](int a) { return bar0 + 8u * (2 * S1 + a); };
  auto acc_full = [&](int b) { return bar0 + 8u * (2 * S1 + S2 + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (2 * S1 + S2 + 2 + b); };
  auto res_full = [&](int w, int b) { return bar0 + 8u * (2 * S1 + S2 + 4 + NB * w + b); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S1 + S2 + 4 + 4 * NB);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L::kOffMisc + 4);
  float* ss_scale = reinterpret_cast<float*>(gbase + L::kOffSS);
  float* ss_shift = ss_scale + BN;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S1; ++s) {
      // gather mode: one cp.async arrival per loader thread; TMA modes: one
      // arrival (with the transaction bytes of A and B) from the issuing thread
      mbar_init(s1_full(s), p.a_mode == kALoadGather ? 128 : 1);
      mbar_init(s1_empty(s), 1);  // the MMA commit (the MMAs ran after the converters)
    }
    // one arrival per converter / epilogue warp (lane 0, after the warp has
    // converged): 128 single-thread arrivals on one barrier serialise for ~1k
    // cycles, which sat on the MMA thread's critical path
    for (int a = 0; a < S2; ++a) mbar_init(t_full(a), 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), kEpiThreads / 32);
    }
    for (int w = 0; w < 4; ++w)
      for (int b = 0; b < NB; ++b) mbar_init(res_full(w, b), 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tm_hi);
    if (L::kSplit) prefetch_tmap(&tm_lo);
    if (p.a_mode != kALoadGather) prefetch_tmap(&tm_a);
    if (p.kb_split) prefetch_tmap(&tm_a2);
    prefetch_tmap(&tm_y);
    if (p.res) prefetch_tmap(&tm_res);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the next kernel on the stream may start its
  // CTAs (barrier set-up, TMEM allocation) on SMs this grid has left, and this
  // grid's prologue above may have overlapped the previous kernel's tail; no
  // global memory is touched before the previous grid has completed and its
  // writes are visible.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int total_tiles = p.m_tiles * p.n_tiles * p.batches;
  // tile t -> (batch, m-tile, n-tile), n fastest: CTAs running together share
  // the A tiles through L2
  auto tile_coords = [&](int t, int& b, int& mt, int& nt) {
    nt = t % p.n_tiles;
    const int r = t / p.n_tiles;
    mt = r % p.m_tiles;
    b = r / p.m_tiles;
  };
  const int my_tiles =
      (blockIdx.x < total_tiles) ? (total_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  // K split (p.ksplit > 1): the problem is run as p.ksplit "batches" over the
  // same A and B, batch b taking k-blocks [b * nkb, (b + 1) * nkb) and storing
  // its raw partial sums to its own slice of y
  const int nkb = p.ksplit > 1 ? p.num_kb / p.ksplit : p.num_kb;
  const int total_items = my_tiles * nkb;
  // The MMAs read A straight from the stage that TMA landed (TF32, bf16
  // activations) and no stage needs rewriting (no taps-mode boxes, no K
  // padding): the MMA thread waits for the stage itself and the converter warps
  // have no work.
  const bool direct = !L::kTmemA && (p.a_mode == kALoadTma2d || p.a_mode == kALoadIm2col) && p.K % kBK == 0;

  if (warp >= kLoadWarp0 && warp < kConvWarp0) {
    // ------------------------------------------------------------ loaders
    const int lt = threadIdx.x - kLoadWarp0 * 32;
    if (p.a_mode != kALoadGather) {
      // lane 0 of each of NL loader warps issues every NL-th stage: the TMA issue
      // path of one thread is slower than the MMAs of one stage.  NL <= S1: a
      // lane's wait for stage use u must never start before use u - 2 has
      // completed, or the parity wait would pass a phase early (the lane last
      // waited for the stage of its previous item, NL items back).
      constexpr int NL = S1 < 4 ? S1 : 4;
      if (lane == 0 && warp - kLoadWarp0 < NL) {
        const int OHW = p.OH * p.OW;
        for (int item = warp - kLoadWarp0; item < total_items; item += NL) {
          const int s = item % S1;
          // Every coordinate of this item's loads is worked out before waiting
          // for its stage: the integer divisions take ~2k cycles, which would
          // otherwise sit between the stage's release and its refill, i.e. on
          // the round trip that bounds the K loop.
          const int tj = item / nkb;
          int b, mt, nt;
          tile_coords(blockIdx.x + tj * gridDim.x, b, mt, nt);
          const int kb = item - tj * nkb + (p.ksplit > 1 ? b * nkb : 0);  // k-block in K
          const int k0 = kb * kBK;
          // A bytes of this k-block: taps beyond K (the zero-weight padding of
          // the last k-block) are not loaded; the converters zero them
          const int a_taps = p.a_mode == kALoadIm2colTaps ? max(0, min(kBK / p.Cs, (p.K - k0) / p.Cs))
                                                          : (k0 < p.K ? 1 : 0);
          const uint32_t a_box = p.a_mode == kALoadIm2colTaps ? kBM * p.Cs * 4 : L::kARaw;
          const uint32_t tx_bytes = a_taps * a_box + (L::kSplit ? 2 : 1) * L::kBBytes;
          const int tap = k0 / p.Cs;
          const int c0 = k0 - tap * p.Cs;
          const uint32_t dst = a_raw + s * L::kARaw;
          int a_r0 = 0, a_x = 0, a_y = 0, a_n = 0;
          uint16_t off_w[kBK / 4], off_h[kBK / 4];  // im2col tap offsets (<= 8 taps per k-block)
          if (p.a_mode == kALoadTma2d) {
            a_r0 = (p.a_off ? (int)(p.a_off[b] / p.Cs) : 0) + p.m_base + mt * kBM;
          } else {
            const int m0 = p.m_base + mt * kBM;
            a_n = m0 / OHW;
            const int rem = m0 - a_n * OHW;
            const int oh0 = rem / p.OW;
            a_x = (rem - oh0 * p.OW) * p.sw - p.pw;
            a_y = oh0 * p.sh - p.ph;
#pragma unroll
            for (int j = 0; j < kBK / 4; ++j) {
              const int r = (tap + j) / p.KW;
              off_w[j] = (uint16_t)((tap + j - r * p.KW) * p.dw);
              off_h[j] = (uint16_t)(r * p.dh);
            }
          }
          const int brow = nt * BN + (p.b_row ? p.b_row[b] : 0);
          // second source (two-source problems): 32 channels of the 1x1 input
          // x2 at the output pixels of this tile
          const bool src2 = p.kb_split && kb >= p.kb_split;
          int b_x = 0, b_y = 0, b_n = 0;
          if (src2 && p.a_mode2 != kALoadTma2d) {
            const int m0 = p.m_base + mt * kBM;
            b_n = m0 / OHW;
            const int rem = m0 - b_n * OHW;
            const int oh0 = rem / p.OW;
            b_x = (rem - oh0 * p.OW) * p.s2;
            b_y = oh0 * p.s2;
          }
          if (!mbar_wait(s1_empty(s), ((item / S1) & 1) ^ 1, abort_flag, p.status)) break;
          mbar_arrive_expect_tx(s1_full(s), tx_bytes);
          if (src2) {
            const int k2 = (kb - p.kb_split) * kBK;
            if (p.a_mode2 == kALoadTma2d)
              tma_load_2d(dst, &tm_a2, k2, p.m_base + mt * kBM, s1_full(s));
            else
              tma_load_im2col_4d(dst, &tm_a2, k2, b_x, b_y, b_n, 0, 0, s1_full(s));
          } else if (p.a_mode == kALoadTma2d) {
            if (a_taps) tma_load_2d(dst, &tm_a, c0, a_r0, s1_full(s));
          } else {
#pragma unroll
            for (int j = 0; j < kBK / 4; ++j)
              if (j < a_taps)
                tma_load_im2col_4d(dst + j * a_box, &tm_a, c0, a_x, a_y, a_n, off_w[j], off_h[j], s1_full(s));
          }
          tma_load_2d(b_hi + s * L::kBStride, &tm_hi, k0, brow, s1_full(s));
          if (L::kSplit) tma_load_2d(b_lo + s * L::kBStride, &tm_lo, k0, brow, s1_full(s));
        }
      }
    } else {
      // thread -> (16-byte chunk c of 8 per row, rows rslot + 16 i)
      const int chunk = lt & 7;
      const int rslot = lt >> 3;
      int pix[8], ih0[8], iw0[8];
      const float* xb = p.x;
      int cur_tile = -1;
      const int OHW = p.OH * p.OW;
      for (int item = 0; item < total_items; ++item) {
        const int s = item % S1;
        if (!mbar_wait(s1_empty(s), ((item / S1) & 1) ^ 1, abort_flag, p.status)) break;
        const int tj = item / nkb;
        int b, mt, nt;
        tile_coords(blockIdx.x + tj * gridDim.x, b, mt, nt);
        const int kb = item - tj * nkb + (p.ksplit > 1 ? b * nkb : 0);
        if (tj != cur_tile) {
          cur_tile = tj;
          xb = p.x + (p.a_off ? p.a_off[b] : 0ll);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int m = mt * kBM + rslot + 16 * i;
            if (m < p.M) {
              const int n = (p.m_base + m) / OHW;
              const int rem = p.m_base + m - n * OHW;
              const int oh = rem / p.OW;
              const int ow = rem - oh * p.OW;
              pix[i] = n * p.Hin * p.Win;
              ih0[i] = oh * p.sh - p.ph;
              iw0[i] = ow * p.sw - p.pw;
            } else {
              pix[i] = 0;
              ih0[i] = -(1 << 28);
              iw0[i] = 0;
            }
          }
        }
        if (lt == 0) {
          const int brow = nt * BN + (p.b_row ? p.b_row[b] : 0);
          mbar_expect_tx(s1_full(s), (L::kSplit ? 2 : 1) * L::kBBytes);
          tma_load_2d(b_hi + s * L::kBStride, &tm_hi, kb * kBK, brow, s1_full(s));
          if (L::kSplit) tma_load_2d(b_lo + s * L::kBStride, &tm_lo, kb * kBK, brow, s1_full(s));
        }
        const int k = kb * kBK + chunk * 4;
        int dy = 0, dx = 0, ci = 0;
        const bool kval = k < p.K;
        if (kval) {
          const int tap = k / p.Cs;
          ci = k - tap * p.Cs;
          const int r = tap / p.KW;
          dy = r * p.dh;
          dx = (tap - r * p.KW) * p.dw;
        }
        const uint32_t stage = a_raw + s * L::kARaw;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = rslot + 16 * i;
          const int ih = ih0[i] + dy, iw = iw0[i] + dx;
          const bool ok = kval && (unsigned)ih < (unsigned)p.Hin && (unsigned)iw < (unsigned)p.Win;
          const float* src =
              ok ? xb + ((long long)pix[i] + (long long)ih * p.Win + iw) * p.Cs + ci : p.x;
          cp_async_16(stage + swz128(row, chunk), src, ok ? 16u : 0u);
        }
        cp_async_arrive_noinc(s1_full(s));
      }
      cp_async_wait_all();
    }
  } else if (warp >= kConvWarp0 && warp < kMmaWarp) {
    // ------------------------------------------------------------ converters
    const int q = warp - kConvWarp0;  // TMEM lane quadrant
    const int row = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    // where the 16-byte chunk c (k offsets 4c..4c+3) of this row sits in a stage:
    // 128-byte swizzled rows, or (taps mode) one [128][Cs] box per filter tap
    uint32_t coff[kBK / 4];
#pragma unroll
    for (int c = 0; c < kBK / 4; ++c)
      coff[c] = p.a_mode == kALoadIm2colTaps
                    ? (uint32_t)((4 * c / p.Cs) * kBM * p.Cs * 4 + row * p.Cs * 4 + (4 * c % p.Cs) * 4)
                    : swz128(row, c);
    const bool taps = p.a_mode == kALoadIm2colTaps;
    int kb = 0, kbase = 0;
    for (int item = 0; item < (direct ? 0 : total_items); ++item) {
      const int s = item % S1;
      const int a = item % S2;
      // decisions stay warp-uniform: lane 0 arrives for the whole warp
      bool ok = __all_sync(0xffffffffu, mbar_wait(s1_full(s), (item / S1) & 1, abort_flag, p.status));
      if constexpr (L::kABf16) {
        // bf16 activations: the MMAs read the stage as it landed (whole taps of
        // 64-channel multiples, no K padding), so there is nothing to convert
        if (!ok) break;
        if (lane == 0) mbar_arrive(t_full(a));
        continue;
      }
      const uint32_t rbase = a_raw + s * L::kARaw;
      // k beyond K: padding of the last k-block (zero weights); never multiply
      // whatever the stage held there
      if (kb == 0 && p.ksplit > 1) {  // first k-block of a tile: its place in K
        int b, mt, nt;
        tile_coords(blockIdx.x + (item / nkb) * gridDim.x, b, mt, nt);
        kbase = b * nkb;
      }
      const int kvalid = p.K - (kbase + kb) * kBK;
      if (++kb == nkb) kb = 0;
      // TF32: the MMAs read the raw fp32 A from shared memory (the tensor core
      // uses the upper 19 bits of the container); the stage is only rewritten
      // when its layout is not the MMA's (taps mode) or padding must be zeroed.
      // 3xTF32: A goes to TMEM, so its shared-memory layout does not matter.
      const bool rewrite = !L::kTmemA && (taps || kvalid < kBK);
      float v[kBK];
      if (ok && (L::kTmemA || rewrite)) {
#pragma unroll
        for (int c = 0; c < kBK / 4; ++c) {
          const float4 f = ld_shared_f4(rbase + coff[c]);
          v[4 * c] = f.x;
          v[4 * c + 1] = f.y;
          v[4 * c + 2] = f.z;
          v[4 * c + 3] = f.w;
        }
      }
      // taps mode rewrites the stage in another layout: every converter has
      // read its row before any writes (the AND keeps an abort uniform)
      if (!L::kTmemA && taps) ok = named_bar_and(ok, 128, 2);
      if (!ok) break;
      if (kvalid < kBK) {
#pragma unroll
        for (int e = 0; e < kBK; ++e)
          if (e >= kvalid) v[e] = 0.f;
      }
      if (rewrite) {
#pragma unroll
        for (int c = 0; c < kBK / 4; ++c)
          st_shared_f4(rbase + swz128(row, c), v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
      }
      if constexpr (L::kBf16 && !L::kABf16) {
        // bf16 pairs (lower k in the low half) into TMEM slot a, once the MMAs of
        // the slot's previous use have completed (see the 3xTF32 case below)
        if (item >= S2) {
          const int prev = item - S2;
          if (!__all_sync(0xffffffffu, mbar_wait(s1_empty(prev % S1), (prev / S1) & 1, abort_flag, p.status)))
            break;
        }
        uint32_t pk[kBK / 2];
#pragma unroll
        for (int e = 0; e < kBK / 2; ++e) {
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
          pk[e] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        tc_fence_after();
        tmem_st_32x32b_x16(tmem_base + lane_addr + L::kACol0 + a * L::kAStageCols, pk);
        tmem_st_wait();
        tc_fence_before();
      }
      if constexpr (L::kSplit) {
        // hi = trunc_tf32(v), lo = rna_tf32(v - hi) into TMEM slot a, once the
        // MMAs of the slot's previous use (item - S2) have completed: their
        // commit is the one that freed that item's shared-memory stage.  No
        // parity ambiguity: the refill this thread saw on s1_full needed the
        // commit of item - S1, and commits complete in order.
        if (item >= S2) {
          const int prev = item - S2;
          if (!__all_sync(0xffffffffu, mbar_wait(s1_empty(prev % S1), (prev / S1) & 1, abort_flag, p.status)))
            break;
        }
        uint32_t hl[kBK];
#pragma unroll
        for (int e = 0; e < kBK; ++e) hl[e] = __float_as_uint(tf32_trunc(v[e]));
        tc_fence_after();
        const uint32_t slot = tmem_base + lane_addr + L::kACol0 + a * L::kAStageCols;
        tmem_st_32x32b_x32(slot, hl);
#pragma unroll
        for (int e = 0; e < kBK; ++e) hl[e] = __float_as_uint(to_tf32(v[e] - tf32_trunc(v[e])));
        tmem_st_32x32b_x32(slot + kBK, hl);
        tmem_st_wait();
        tc_fence_before();
      }
      if (rewrite) fence_proxy_async_smem();  // the generic-proxy stores, visible to the tensor core
      __syncwarp();  // every lane's TMEM / shared-memory stores precede lane 0's arrival
      if (lane == 0) mbar_arrive(t_full(a));
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // One thread issues every MMA of the CTA, walking its k-blocks with
    // incremental ring indices: the issue rate of this thread bounds the kernel.
    constexpr uint32_t idesc = make_idesc(2, kBM, BN);
    constexpr uint32_t idesc2 = make_idesc(2, kBM, 2 * BN);  // stacked B (BN = 64)
    constexpr uint32_t idesc_bf = make_idesc(1, kBM, BN);    // bf16 x bf16
    if (lane == 0) {
      bool issued = false, ok = true;
      uint32_t cc = 0;             // accumulation units started (chunks / tiles)
      int s = 0, a = 0;            // shared-memory stage, TMEM A slot
      uint32_t pa = 0;             // parity of slot a's current use
      int kb = 0;                  // k-block in the tile
      // One accumulation unit (a chunk of kChunkKB k-blocks, or a whole tile
      // when the accumulator is not promoted) per outer iteration; the inner
      // loop is unrolled so that its k-blocks run without a loop back-edge or
      // bookkeeping between them (those cost ~400 cycles of this thread's time
      // per k-block, and this thread's issue rate bounds the kernel).
      for (int item = 0; ok && item < total_items;) {
        const int cb = cc & 1;
        if (!mbar_wait(acc_empty(cb), ((cc >> 1) & 1) ^ 1, abort_flag, p.status)) break;
        const uint32_t d_tmem = tmem_base + (L::kPromote ? L::kChunkCols * (1 + cb) : BN * cb);
        const int len = L::kPromote ? min(L::kChunkKB, nkb - kb) : nkb - kb;
        constexpr int kU = 4;  // k-blocks per unrolled group
        static_assert(!L::kPromote || L::kChunkKB % kU == 0, "whole unrolled groups per chunk");
        for (int k0 = 0; ok && k0 < len; k0 += kU) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int kin = k0 + u;
          if (kin >= len) break;
          // the converters arrive on t_full only after they saw the stage's TMA
          // (A and B) complete on s1_full and wrote its A operands
          if (direct ? !mbar_wait(s1_full(s), (item / S1) & 1, abort_flag, p.status)
                     : !mbar_wait(t_full(a), pa, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ahi = tmem_base + L::kACol0 + a * L::kAStageCols;  // 3xTF32: A hi | lo
          const uint32_t alo = ahi + kBK;
          const uint64_t da = smem_desc_sw128(a_raw + s * L::kARaw);  // TF32: A as landed
          const uint64_t dbh = (L::kBf16 && !L::kABf16) ? smem_desc_sw64(b_hi + s * L::kBStride)
                                                         : smem_desc_sw128(b_hi + s * L::kBStride);
          uint64_t dbl = 0;
          if constexpr (L::kSplit) dbl = smem_desc_sw128(b_lo + s * L::kBStride);
          if constexpr (L::kABf16) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)  // A and B from shared memory, 128-byte rows
              tc_mma<1>(d_tmem, da + (uint64_t)(kk * 2), dbh + (uint64_t)(kk * 2), idesc_bf, (kin | kk) ? 1u : 0u);
          } else if constexpr (L::kBf16) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)  // K = 16 bf16 (32 bytes) per MMA
              tc_mma_f16_ts(d_tmem, ahi + kk * 8, dbh + (uint64_t)(kk * 2), idesc_bf, (kin | kk) ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < (L::kBf16 ? 0 : kBK / 8); ++kk) {
            const uint32_t acc = (kin | kk) ? 1u : 0u;
            if constexpr (L::kStack) {
              // [hi.b_hi | hi.b_lo] over B hi and B lo rows, then lo.b_hi into the
              // second (small-term) half
              tc_mma_tf32_ts(d_tmem, ahi + kk * 8, dbh + (uint64_t)(kk * 2), idesc2, acc);
              tc_mma_tf32_ts(d_tmem + BN, alo + kk * 8, dbh + (uint64_t)(kk * 2), idesc, 1u);
            } else if constexpr (L::kSplit) {
              tc_mma_tf32_ts(d_tmem, ahi + kk * 8, dbh + (uint64_t)(kk * 2), idesc, acc);
              tc_mma_tf32_ts(d_tmem, ahi + kk * 8, dbl + (uint64_t)(kk * 2), idesc, 1u);
              tc_mma_tf32_ts(d_tmem, alo + kk * 8, dbh + (uint64_t)(kk * 2), idesc, 1u);
            } else {
              tc_mma<0>(d_tmem, da + (uint64_t)(kk * 2), dbh + (uint64_t)(kk * 2), idesc, acc);
            }
          }
          // frees the shared-memory stage (and, through it, the TMEM A slot: the
          // converters wait for this commit before refilling the slot)
          tc_commit(s1_empty(s));
          issued = true;
          ++item;
          if (++s == S1) s = 0;
          if (++a == S2) {
            a = 0;
            pa ^= 1;
          }
        }
        }
        if (!ok) break;
        kb += len;
        if (kb == nkb) kb = 0;
        tc_commit(acc_full(cb));
        ++cc;
      }
      // every MMA issued by this thread completes before TMEM is freed
      if (issued) {
        tc_commit(drain_bar);
        volatile int no_abort = 0;
        mbar_wait(drain_bar, 0, &no_abort, p.status);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Each warp stores (and loads the residual of) its own 32 rows of a group
    // with its own TMA boxes, so groups need no barrier across the four warps;
    // the warps agree (barrier AND-reduction) only once per accumulator chunk
    // and per tile, which also keeps every abort decision uniform.
    const int et = threadIdx.x;  // 0..127 = tile row
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    constexpr int kWTile = kEpiTile / 4;  // this warp's 32 rows of a staging tile
    uint32_t cc = 0;   // accumulator chunks consumed
    uint32_t grp = 0;  // kEG-column output groups produced (staging buffer = grp % NB)
    bool ok = true;
    // lane 0: residual loads issued but not yet waited for (per buffer), so an
    // abort can let them land before the CTA exits
    uint32_t res_out = 0, res_par[NB] = {};
    auto issue_res = [&](uint32_t g, int col, int r0, int b) {
      const int rb = g % NB;
      mbar_arrive_expect_tx(res_full(warp, rb), kWTile);
      tma_load_3d(res_st + rb * kEpiTile + warp * kWTile, &tm_res, col, r0, b, res_full(warp, rb));
      res_out |= 1u << rb;
      res_par[rb] = (g / NB) & 1;
    };
    for (int tj = 0; tj < my_tiles; ++tj) {
      int b, mt, nt;
      tile_coords(blockIdx.x + tj * gridDim.x, b, mt, nt);
      const int m0 = mt * kBM;
      const int r0 = m0 + warp * 32;        // this warp's first row
      const bool rows_in = r0 < p.M;        // boxes entirely past M are skipped
      const int rem_cols = p.Nc - nt * BN;
      const int ngroups = rem_cols >= BN ? BN / kEG : (rem_cols + kEG - 1) / kEG;
      // all four warps are done with the previous tile (and its staged scale /
      // shift); an abort in any of them ends the loop for all
      ok = named_bar_and(ok, kEpiThreads);
      if (!ok) break;
      // this tile's per-channel scale / shift, staged once in shared memory
      if (p.scale || p.shift) {
        for (int c = et; c < BN; c += kEpiThreads) {
          const int gc = nt * BN + c;
          ss_scale[c] = (p.scale && gc < p.Nc) ? p.scale[gc] : 1.f;
          ss_shift[c] = (p.shift && gc < p.Nc) ? p.shift[gc] : 0.f;
        }
        named_bar_sync(kEpiThreads);
      }
      // residual blocks of the first NB groups (later ones after each use)
      if (p.res && lane == 0 && rows_in) {
        for (int g = 0; g < NB && g < ngroups; ++g) issue_res(grp + g, nt * BN + g * kEG, r0, b);
      }
      const int nch = L::kPromote ? (nkb + L::kChunkKB - 1) / L::kChunkKB : 1;
      for (int ch = 0; ch < nch; ++ch) {
        const int cb = L::kPromote ? (cc & 1) : (tj & 1);
        const uint32_t cpar = L::kPromote ? ((cc >> 1) & 1) : ((tj >> 1) & 1);
        ok = named_bar_and(ok && mbar_wait(acc_full(cb), cpar, abort_flag, p.status), kEpiThreads);
        if (!ok) break;
        tc_fence_after();
        const bool last = ch == nch - 1;
        const uint32_t ccol = L::kPromote ? L::kChunkCols * (1 + cb) : cb * BN;  // accumulator columns
        // Promoted accumulators: every chunk, the tile's last one included, is
        // folded into the running total and its accumulator handed back to the
        // MMA thread at once; the output groups are then produced from the total,
        // so the next tile's MMAs do not wait for this tile's stores.
        if (L::kStack) {
          // total += big + small, 16 columns at a time
          for (int c = 0; c < BN; c += 16) {
            uint32_t a0[16], s0[16], b0[16];
            tmem_ld_32x32b_x16(tmem_base + lane_addr + ccol + c, a0);
            tmem_ld_32x32b_x16(tmem_base + lane_addr + ccol + BN + c, s0);
            if (ch > 0) tmem_ld_32x32b_x16(tmem_base + lane_addr + c, b0);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float v = __uint_as_float(a0[e]) + __uint_as_float(s0[e]);
              if (ch > 0) v = __uint_as_float(b0[e]) + v;
              a0[e] = __float_as_uint(v);
            }
            tmem_st_32x32b_x16(tmem_base + lane_addr + c, a0);
          }
        } else if (L::kPromote) {
          // fold the chunk into the running total: each TMEM round trip carries
          // 32 columns of the chunk and 32 of the total (loads issued before
          // one wait), in 16-column pieces to bound live registers
          const int ncols = (ngroups * kEG + 31) / 32 * 32;  // columns < BN
          for (int c = 0; c < ncols; c += 32) {
            uint32_t a0[16], a1[16], b0[16], b1[16];
            tmem_ld_32x32b_x16(tmem_base + lane_addr + ccol + c, a0);
            tmem_ld_32x32b_x16(tmem_base + lane_addr + ccol + c + 16, a1);
            if (ch > 0) {
              tmem_ld_32x32b_x16(tmem_base + lane_addr + c, b0);
              tmem_ld_32x32b_x16(tmem_base + lane_addr + c + 16, b1);
            }
            tmem_ld_wait();
            if (ch > 0) {
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                a0[e] = __float_as_uint(__uint_as_float(b0[e]) + __uint_as_float(a0[e]));
                a1[e] = __float_as_uint(__uint_as_float(b1[e]) + __uint_as_float(a1[e]));
              }
            }
            tmem_st_32x32b_x16(tmem_base + lane_addr + c, a0);
            tmem_st_32x32b_x16(tmem_base + lane_addr + c + 16, a1);
          }
        }
        if (L::kPromote) {
          tmem_st_wait();  // the folded total is in TMEM
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty(cb));
        }
        // one output group: the running total (promoted) or the tile's
        // accumulator, columns [j * kEG, (j + 1) * kEG), in registers r
        const uint32_t gcol = L::kPromote ? 0u : ccol;
        auto out_group = [&](int j, const uint32_t (&r)[kEG]) -> bool {
          // ---- final values of this group
            const int col0 = nt * BN + j * kEG;
            const int buf = grp % NB;
            float v[kEG];
#pragma unroll
            for (int e = 0; e < kEG; ++e) v[e] = __uint_as_float(r[e]);
#pragma unroll
            for (int q4 = 0; q4 < kEG / 4; ++q4) {
              const int c = j * kEG + 4 * q4;  // column within the tile
              if (p.scale) {
                const float4 sc = *reinterpret_cast<const float4*>(ss_scale + c);
                v[4 * q4] *= sc.x; v[4 * q4 + 1] *= sc.y; v[4 * q4 + 2] *= sc.z; v[4 * q4 + 3] *= sc.w;
              }
              if (p.shift) {
                const float4 sh = *reinterpret_cast<const float4*>(ss_shift + c);
                v[4 * q4] += sh.x; v[4 * q4 + 1] += sh.y; v[4 * q4 + 2] += sh.z; v[4 * q4 + 3] += sh.w;
              }
            }
            bool w = true;
            if (p.res && rows_in) {
              w = mbar_wait(res_full(warp, buf), (grp / NB) & 1, abort_flag, p.status);
              if (w && lane == 0) res_out &= ~(1u << buf);
              if constexpr (L::kOBf16) {
#pragma unroll
                for (int q8 = 0; q8 < kEG / 8; ++q8) {
                  const uint4 rv = lds_u4(res_st + buf * kEpiTile + swz_eg<L::kEpiRow>(et, q8));
                  v[8 * q8] += bf16_lo(rv.x); v[8 * q8 + 1] += bf16_hi(rv.x);
                  v[8 * q8 + 2] += bf16_lo(rv.y); v[8 * q8 + 3] += bf16_hi(rv.y);
                  v[8 * q8 + 4] += bf16_lo(rv.z); v[8 * q8 + 5] += bf16_hi(rv.z);
                  v[8 * q8 + 6] += bf16_lo(rv.w); v[8 * q8 + 7] += bf16_hi(rv.w);
                }
              } else {
#pragma unroll
                for (int q4 = 0; q4 < kEG / 4; ++q4) {
                  const float4 rv = ld_shared_f4(res_st + buf * kEpiTile + swz_eg<L::kEpiRow>(et, q4));
                  v[4 * q4] += rv.x; v[4 * q4 + 1] += rv.y; v[4 * q4 + 2] += rv.z; v[4 * q4 + 3] += rv.w;
                }
              }
            }
            if (p.relu) {
#pragma unroll
              for (int e = 0; e < kEG; ++e) v[e] = v[e] > 0.f ? v[e] : 0.f;
            }
            // this warp's staging rows of NB groups ago must have been read by its
            // TMA store (the warp vote below also orders lane 0's wait first)
            if (lane == 0) bulk_wait_group_read<NB - 1>();
            if (!__all_sync(0xffffffffu, w)) {
              return false;  // decided with the other warps at the next barrier
            }
            const uint32_t ost = out_st + buf * kEpiTile;
            if constexpr (L::kOBf16) {
#pragma unroll
              for (int q8 = 0; q8 < kEG / 8; ++q8)
                sts_u4(ost + swz_eg<L::kEpiRow>(et, q8), pack_bf16x2(v[8 * q8], v[8 * q8 + 1]),
                       pack_bf16x2(v[8 * q8 + 2], v[8 * q8 + 3]), pack_bf16x2(v[8 * q8 + 4], v[8 * q8 + 5]),
                       pack_bf16x2(v[8 * q8 + 6], v[8 * q8 + 7]));
            } else {
#pragma unroll
              for (int q4 = 0; q4 < kEG / 4; ++q4)
                sts_v4(ost + swz_eg<L::kEpiRow>(et, q4), v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && rows_in) {
              tma_store_3d(&tm_y, col0, r0, b, ost + warp * kWTile);
              bulk_commit_group();
              if (p.res && j + NB < ngroups) issue_res(grp + NB, col0 + NB * kEG, r0, b);  // freed buffer
            }
            ++grp;
            return true;
        };
        if (kEG > 16 && last) {
          // 32-column groups: one TMEM round trip per group (two groups' worth of
          // registers would spill at the 128 registers a 416-thread block gets)
          for (int j = 0; j < ngroups; ++j) {
            uint32_t r[kEG];
            tmem_ld_cols(tmem_base + lane_addr + gcol + j * kEG, r);
            tmem_ld_wait();
            if (!out_group(j, r)) { ok = false; break; }
          }
        } else if (last && ngroups > 0) {
          // the TMEM load of group j + 1 is in flight while group j is scaled,
          // staged and stored
          uint32_t ra[kEG], rb[kEG];
          tmem_ld_cols(tmem_base + lane_addr + gcol, ra);
          tmem_ld_wait();
          for (int j = 0; j < ngroups; j += 2) {
            if (j + 1 < ngroups) tmem_ld_cols(tmem_base + lane_addr + gcol + (j + 1) * kEG, rb);
            const bool g_ok = out_group(j, ra);
            tmem_ld_wait();
            if (!g_ok) { ok = false; break; }
            if (j + 1 >= ngroups) break;
            if (j + 2 < ngroups) tmem_ld_cols(tmem_base + lane_addr + gcol + (j + 2) * kEG, ra);
            const bool g_ok2 = out_group(j + 1, rb);
            tmem_ld_wait();
            if (!g_ok2) { ok = false; break; }
          }
        }
        if (!L::kPromote) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty(cb));
        }
        if (L::kPromote) ++cc;
      }
    }
    if (lane == 0) {
      bulk_wait_group<0>();  // stores complete before the CTA exits
      for (int rb = 0; rb < NB; ++rb)
        if (res_out & (1u << rb)) {  // only after an abort
          volatile int no_abort = 0;
          mbar_wait(res_full(warp, rb), res_par[rb], &no_abort, p.status);
        }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

typedef CUresult (*EncodeTiledFn3)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn3 tiled_fn() {
  static EncodeTiledFn3 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiledFn3>(f);
  }();
  return fn;
}

// [batches][rows][cols] output / residual (fp32, or bf16 when es == 2) with
// row stride ld, batch stride bstride (elements); 32-row x eg boxes (one per
// epilogue warp), 64- or 128-byte rows with the matching swizzle.
int encode_out_map(const void* base, int cols, int rows, int batches, int ld, long long bstride,
                   int eg, int es_bytes, CUtensorMap* map) {
  EncodeTiledFn3 fn = tiled_fn();
  if (!fn) return (int)CUDA_ERROR_NOT_FOUND;
  const long long bs = batches > 1 ? bstride : (long long)rows * ld;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batches};
  cuuint64_t strides[2] = {(cuuint64_t)ld * es_bytes, (cuuint64_t)bs * es_bytes};
  cuuint32_t box[3] = {(cuuint32_t)eg, 32u, 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  return (int)fn(map, es_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                 const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 eg * es_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int PREC, int BN, int EG, int NB, int AIO = 0>
int launch3_t(const IgemmParams& p, const CUtensorMap& hi, const CUtensorMap& lo,
              const CUtensorMap& am, const CUtensorMap& am2, int num_sms, cudaStream_t st) {
  using L = Layout<PREC, BN, EG, NB, AIO>;
  // the shared-memory opt-in is a per-device attribute of the kernel
  constexpr int kMaxDevices = 64;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(igemm_tc3_kernel<PREC, BN, EG, NB, AIO>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return (int)e;
    attr_set[dev] = true;
  }
  CUtensorMap ym{}, rm{};
  int er = encode_out_map(p.y, p.Nc, p.M, p.batches, p.ldy, p.y_bstride, EG, L::kOes, &ym);
  if (er) return (int)cudaErrorInvalidValue;
  if (p.res) {
    er = encode_out_map(p.res, p.Nc, p.M, p.batches, p.ldr, p.y_bstride, EG, L::kOes, &rm);
    if (er) return (int)cudaErrorInvalidValue;
  }
  const int total = p.m_tiles * p.n_tiles * p.batches;
  const int grid = total < num_sms ? total : num_sms;
  if (grid <= 0) return 0;
  // Launched as a programmatic dependent of the previous kernel on the stream
  // (the kernel waits for it before touching global memory).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, igemm_tc3_kernel<PREC, BN, EG, NB, AIO>, p, hi, lo, am, am2, ym, rm);
}

}  // namespace

constexpr int kLongK = 16;  // k-blocks (K >= 512)
constexpr int kShortK = 2;  // k-blocks (K <= 64)

int igemm3_launch(const IgemmParams& p, const CUtensorMap& hi, const CUtensorMap& lo,
                  const CUtensorMap& am, const CUtensorMap& am2, int precision, int bn, int num_sms,
                  cudaStream_t st) {
  // 3xTF32, BN = 128: 16-column epilogue groups buy a fourth operand stage,
  // worth it once the K loop of a tile is long (short-K layers are bound by
  // their epilogue, which 32-column groups store faster)
  // Short K loops are bound by the epilogue's HBM traffic: four staging
  // buffers (more stores and residual loads in flight) instead of operand stages.
  const int kb_tile = p.ksplit > 1 ? p.num_kb / p.ksplit : p.num_kb;  // k-blocks per tile
  const bool short_k = kb_tile <= kShortK;
  if (precision == kPrec3xTF32 && bn == 64)
    return short_k ? launch3_t<kPrec3xTF32, 64, 32, 4>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrec3xTF32, 64, 32, 2>(p, hi, lo, am, am2, num_sms, st);
  if (precision == kPrec3xTF32 && bn == 128)
    return kb_tile >= kLongK ? launch3_t<kPrec3xTF32, 128, 16, 2>(p, hi, lo, am, am2, num_sms, st)
           : short_k          ? launch3_t<kPrec3xTF32, 128, 32, 4>(p, hi, lo, am, am2, num_sms, st)
                              : launch3_t<kPrec3xTF32, 128, 32, 2>(p, hi, lo, am, am2, num_sms, st);
  if (precision == kPrecTF32 && bn == 64)
    return short_k ? launch3_t<kPrecTF32, 64, 32, 4>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecTF32, 64, 32, 2>(p, hi, lo, am, am2, num_sms, st);
  if (precision == kPrecTF32 && bn == 128)
    return short_k ? launch3_t<kPrecTF32, 128, 32, 4>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecTF32, 128, 32, 2>(p, hi, lo, am, am2, num_sms, st);
  if (precision == kPrecTF32 && bn == 256) return launch3_t<kPrecTF32, 256, 32, 2>(p, hi, lo, am, am2, num_sms, st);
  // bf16 activations (AIO bit 0) and / or bf16 outputs (bit 1)
  const int aio = (p.a_bf16 ? 1 : 0) | (p.out_bf16 ? 2 : 0);
  if (aio && precision != kPrecBF16) return (int)cudaErrorInvalidValue;
  if (aio == 3 && bn == 256 && !short_k) return launch3_t<kPrecBF16, 256, 32, 2, 3>(p, hi, lo, am, am2, num_sms, st);
  if (aio == 3 && bn == 64)
    return short_k ? launch3_t<kPrecBF16, 64, 32, 4, 3>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecBF16, 64, 32, 2, 3>(p, hi, lo, am, am2, num_sms, st);
  if (aio == 3 && bn == 128)
    return short_k ? launch3_t<kPrecBF16, 128, 32, 4, 3>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecBF16, 128, 32, 2, 3>(p, hi, lo, am, am2, num_sms, st);
  if (aio == 2 && bn == 64)
    return short_k ? launch3_t<kPrecBF16, 64, 32, 4, 2>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecBF16, 64, 32, 2, 2>(p, hi, lo, am, am2, num_sms, st);
  if (aio == 2 && bn == 128)
    return short_k ? launch3_t<kPrecBF16, 128, 32, 4, 2>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecBF16, 128, 32, 2, 2>(p, hi, lo, am, am2, num_sms, st);
  if (aio) return (int)cudaErrorInvalidValue;
  if (precision == kPrecBF16 && bn == 64)
    return short_k ? launch3_t<kPrecBF16, 64, 32, 4>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecBF16, 64, 32, 2>(p, hi, lo, am, am2, num_sms, st);
  if (precision == kPrecBF16 && bn == 128)
    return short_k ? launch3_t<kPrecBF16, 128, 32, 4>(p, hi, lo, am, am2, num_sms, st)
                   : launch3_t<kPrecBF16, 128, 32, 2>(p, hi, lo, am, am2, num_sms, st);
  return (int)cudaErrorInvalidValue;
}

}  // namespace ob2
