// tcgen05 / TMEM implicit-GEMM kernel for sm_100a: convolution (no im2col
// buffer) and batched broadcast GEMM share it.
//
// Replaces the reference's compute_conv2d_im2col + im2col_2d
// (src/ops/nn/conv.rs:1142-1368), its direct 1x1 path (conv.rs:849-935 via the
// SIMD strategy), compute_matmul's per-batch sgemm (src/ops/math/matmul.rs:124-279)
// and compute_gemm (src/ops/math/gemm.rs:172-291).
//
// Persistent, warp-specialised, one CTA per SM:
//   warps 0-3      epilogue: TMEM -> registers (tcgen05.ld), scale/shift,
//                  residual, relu, global store.  Warp w owns TMEM lanes 32w..32w+31.
//   warps 4..4+4G  A producers in G groups of 128 threads; group g fills the
//                  k-blocks with index = g (mod G).  Each thread gathers 16-byte
//                  chunks of NHWC activations straight from global memory (zero
//                  fill for padding), splits them into tf32 hi/lo (3xTF32) or
//                  rounds them (tf32 / bf16), and stores them in the 128-byte
//                  (64-byte for bf16) swizzled K-major layout.  Thread 0 of the
//                  group also issues the TMA loads of the weight tiles.
//   last warp      TMEM allocation and the single-thread tcgen05.mma issue.
// Accumulators: two TMEM buffers of BN fp32 columns, so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// 3xTF32: a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi with hi = rna_tf32(v),
// lo = rna_tf32(v - hi) (split-precision scheme of Ootomo & Yokota, 2022).
// Weights are split once when packed; activations are split by the producers.
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace ob2 {

namespace {

constexpr int kBM = 128;
constexpr int kEpiWarps = 4;
constexpr int kGroups = 2;               // producer groups
constexpr int kProdThreads = 128;        // threads per producer group
constexpr int kProdWarps = kGroups * kProdThreads / 32;
constexpr int kMmaWarp = kEpiWarps + kProdWarps;
constexpr int kThreads = (kMmaWarp + 1) * 32;
constexpr int kSmemBudget = 200 * 1024;

template <int PREC>
struct Cfg {
  static constexpr bool kSplit = (PREC == kPrec3xTF32);
  static constexpr int kRowBytes = (PREC == kPrecBF16) ? 64 : 128;   // bytes of one A/B row per k-block
  static constexpr int kChunksPerRow = kRowBytes / 16;
  static constexpr int kRowsPerThread = kBM * kChunksPerRow / kProdThreads;  // 8 (tf32) / 4 (bf16)
  static constexpr int kLoadsPerChunk = (PREC == kPrecBF16) ? 2 : 1;        // float4 loads per chunk
  static constexpr int kElemsPerChunk = 4 * kLoadsPerChunk;
  static constexpr int kABytes = kBM * kRowBytes;                          // one A operand tile
  static constexpr int kKSteps = (PREC == kPrecBF16) ? 2 : 4;              // MMAs (K) per k-block
  static constexpr uint32_t kDescStep = 2;                                 // 32 bytes >> 4
};

template <int PREC, int BN>
struct Layout {
  using C = Cfg<PREC>;
  static constexpr int kBBytes = BN * C::kRowBytes;
  static constexpr int kStageBytes = (C::kSplit ? 2 : 1) * (C::kABytes + kBBytes);
  static constexpr int kStagesRaw = kSmemBudget / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kAHi = 0;
  static constexpr int kALo = kAHi + kStages * C::kABytes;
  static constexpr int kBHi = kALo + (C::kSplit ? kStages * C::kABytes : 0);
  static constexpr int kBLo = kBHi + kStages * kBBytes;
  static constexpr int kBar = kBLo + (C::kSplit ? kStages * kBBytes : 0);
  // full[S], empty[S], tfull[2], tempty[2], drain
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int kMisc = kBar + kNumBars * 8;   // tmem base (4B) + abort flag (4B)
  static constexpr int kBytes = kMisc + 16 + 1024;    // + alignment slack
  // 3xTF32 "promotion": the tensor core adds into its fp32 accumulator with
  // truncation, so a long K-loop into one accumulator drifts by ~1 ulp per MMA.
  // In 3xTF32 mode each accumulator therefore only sums kChunkKB k-blocks
  // (24 MMAs); the epilogue warps fold the chunks into a running total with
  // round-to-nearest adds.  TMEM: total [0, BN), chunks [BN, 2BN) and [2BN, 3BN).
  // Other modes: two whole-tile accumulators [0, BN) and [BN, 2BN).
  static constexpr bool kPromote = (PREC == kPrec3xTF32);
  static constexpr int kChunkKB = kPromote ? 2 : (1 << 30);
  static constexpr int kCols = kPromote ? 3 * BN : 2 * BN;
  static constexpr int kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128
                                   : kCols <= 256 ? 256 : 512;
  static_assert(kCols <= 512, "accumulators exceed TMEM");
};

__device__ __forceinline__ uint32_t swz_off(int row, int chunk, int row_bytes) {
  if (row_bytes == 128) return row * 128 + ((chunk ^ (row & 7)) << 4);
  return row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ float4 ldg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Epilogue of 32 consecutive columns of one output row: y = acc * scale + shift
// (+ residual) (relu), float4 stores.
__device__ __forceinline__ void store_row32(const IgemmParams& p, const uint32_t (&r)[32], int col0,
                                            float* yrow, const float* rrow) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int c = col0 + 4 * q;
    if (c < p.Nc) {
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = __uint_as_float(r[4 * q + e]);
      if (p.scale) {
        const float4 sc = *reinterpret_cast<const float4*>(p.scale + c);
        v[0] *= sc.x; v[1] *= sc.y; v[2] *= sc.z; v[3] *= sc.w;
      }
      if (p.shift) {
        const float4 sh = *reinterpret_cast<const float4*>(p.shift + c);
        v[0] += sh.x; v[1] += sh.y; v[2] += sh.z; v[3] += sh.w;
      }
      if (rrow) {
        const float4 rv = *reinterpret_cast<const float4*>(rrow + c);
        v[0] += rv.x; v[1] += rv.y; v[2] += rv.z; v[3] += rv.w;
      }
      if (p.relu) {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = v[e] > 0.f ? v[e] : 0.f;
      }
      *reinterpret_cast<float4*>(yrow + c) = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}

template <int PREC, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    igemm_tc_kernel(const __grid_constant__ IgemmParams p, const __grid_constant__ CUtensorMap tm_hi,
                    const __grid_constant__ CUtensorMap tm_lo) {
  using C = Cfg<PREC>;
  using L = Layout<PREC, BN>;
  constexpr int S = L::kStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_addr);

  const uint32_t a_hi = base + L::kAHi, a_lo = base + L::kALo;
  const uint32_t b_hi = base + L::kBHi, b_lo = base + L::kBLo;
  const uint32_t bar0 = base + L::kBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * S + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * S + 2 + b); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), kProdThreads);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), kEpiWarps * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tm_hi);
    if (C::kSplit) prefetch_tmap(&tm_lo);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = p.m_tiles * p.n_tiles * p.batches;
  // tile t -> (batch, m-tile, n-tile); n fastest so CTAs running together
  // share A tiles through L2.
  auto tile_coords = [&](int t, int& b, int& mt, int& nt) {
    nt = t % p.n_tiles;
    int r = t / p.n_tiles;
    mt = r % p.m_tiles;
    b = r / p.m_tiles;
  };
  const int my_tiles =
      (blockIdx.x < total_tiles) ? (total_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int total_items = my_tiles * p.num_kb;

  if (warp >= kEpiWarps && warp < kMmaWarp) {
    // ------------------------------------------------------------ producers
    const int pw = warp - kEpiWarps;
    const int group = pw / (kProdThreads / 32);
    const int pt = threadIdx.x - (kEpiWarps + group * (kProdThreads / 32)) * 32;
    const int chunk = pt % C::kChunksPerRow;
    const int rslot = pt / C::kChunksPerRow;
    constexpr int kRowStride = kProdThreads / C::kChunksPerRow;  // rows between a thread's rows
    constexpr int R = C::kRowsPerThread;
    constexpr int NL = C::kLoadsPerChunk;

    int pix[R], ih0[R], iw0[R];
    const float* xb = p.x;
    int loaded_tile = -1;
    const int OHW = p.OH * p.OW;

    auto prep_rows = [&](int tj) {
      int b, mt, nt;
      tile_coords(blockIdx.x + tj * gridDim.x, b, mt, nt);
      xb = p.x + (p.a_off ? p.a_off[b] : 0ll);
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int m = mt * kBM + rslot + kRowStride * i;
        if (m < p.M) {
          const int n = m / OHW;
          const int rem = m - n * OHW;
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
    };

    auto load_item = [&](int item, float4 (&v)[R][NL]) {
      const int tj = item / p.num_kb;
      const int kb = item - tj * p.num_kb;
      if (tj != loaded_tile) {
        prep_rows(tj);
        loaded_tile = tj;
      }
#pragma unroll
      for (int h = 0; h < NL; ++h) {
        const int k = kb * (C::kRowBytes / (PREC == kPrecBF16 ? 2 : 4)) + chunk * C::kElemsPerChunk + 4 * h;
        int dy = 0, dx = 0, ci = 0;
        const bool kval = k < p.K;
        if (kval) {
          const int tap = k / p.Cs;
          ci = k - tap * p.Cs;
          const int r = tap / p.KW;
          dy = r * p.dh;
          dx = (tap - r * p.KW) * p.dw;
        }
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const int ih = ih0[i] + dy, iw = iw0[i] + dx;
          if (kval && (unsigned)ih < (unsigned)p.Hin && (unsigned)iw < (unsigned)p.Win) {
            const long long off = ((long long)pix[i] + (long long)ih * p.Win + iw) * p.Cs + ci;
            v[i][h] = ldg_f4(xb + off);
          } else {
            v[i][h] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
    };

    float4 cur[R][NL], nxt[R][NL];
    int item = group;
    if (item < total_items) load_item(item, cur);
    bool ok = true;
    while (item < total_items) {
      const int nitem = item + kGroups;
      if (nitem < total_items) load_item(nitem, nxt);
      const int s = item % S;
      const uint32_t ph = (item / S) & 1;
      if (!mbar_wait(empty_bar(s), ph ^ 1, abort_flag, p.status)) {
        ok = false;
        break;
      }
      if (pt == 0) {
        const int tj = item / p.num_kb;
        const int kb = item - tj * p.num_kb;
        int b, mt, nt;
        tile_coords(blockIdx.x + tj * gridDim.x, b, mt, nt);
        const int brow = nt * BN + (p.b_row ? p.b_row[b] : 0);
        const int kc = kb * (C::kRowBytes / (PREC == kPrecBF16 ? 2 : 4));
        mbar_expect_tx(full_bar(s), (C::kSplit ? 2 : 1) * L::kBBytes);
        tma_load_2d(b_hi + s * L::kBBytes, &tm_hi, kc, brow, full_bar(s));
        if (C::kSplit) tma_load_2d(b_lo + s * L::kBBytes, &tm_lo, kc, brow, full_bar(s));
      }
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const uint32_t off = swz_off(rslot + kRowStride * i, chunk, C::kRowBytes);
        if constexpr (PREC == kPrecBF16) {
          const float4 u = cur[i][0], w = cur[i][NL - 1];
          st_shared_v4(a_hi + s * C::kABytes + off, pack_bf16(u.x, u.y), pack_bf16(u.z, u.w),
                       pack_bf16(w.x, w.y), pack_bf16(w.z, w.w));
        } else {
          const float4 u = cur[i][0];
          const float hx = to_tf32(u.x), hy = to_tf32(u.y), hz = to_tf32(u.z), hw = to_tf32(u.w);
          st_shared_v4(a_hi + s * C::kABytes + off, __float_as_uint(hx), __float_as_uint(hy),
                       __float_as_uint(hz), __float_as_uint(hw));
          if constexpr (C::kSplit) {
            st_shared_v4(a_lo + s * C::kABytes + off, __float_as_uint(to_tf32(u.x - hx)),
                         __float_as_uint(to_tf32(u.y - hy)), __float_as_uint(to_tf32(u.z - hz)),
                         __float_as_uint(to_tf32(u.w - hw)));
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(full_bar(s));
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int h = 0; h < NL; ++h) cur[i][h] = nxt[i][h];
      item = nitem;
    }
    (void)ok;
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = make_idesc(PREC == kPrecBF16 ? 1 : 2, kBM, BN);
    int item = 0;
    bool issued = false;
    uint32_t cc = 0;  // accumulator-chunk counter (3xTF32 promotion)
    for (int tj = 0; tj < my_tiles; ++tj) {
      const int buf = tj & 1;
      const uint32_t aph = (tj >> 1) & 1;
      uint32_t d_tmem = tmem_base + buf * BN;
      int cb = 0;
      if constexpr (!L::kPromote) {
        if (!mbar_wait(tempty_bar(buf), aph ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
      }
      bool failed = false;
      for (int kb = 0; kb < p.num_kb; ++kb, ++item) {
        const int s = item % S;
        const uint32_t ph = (item / S) & 1;
        const int kin = kb % L::kChunkKB;  // k-block index inside the accumulator chunk
        if constexpr (L::kPromote) {
          if (kin == 0) {
            cb = cc & 1;
            if (!mbar_wait(tempty_bar(cb), ((cc >> 1) & 1) ^ 1, abort_flag, p.status)) {
              failed = true;
              break;
            }
            tc_fence_after();
            d_tmem = tmem_base + BN * (1 + cb);
          }
        }
        if (!mbar_wait(full_bar(s), ph, abort_flag, p.status)) {
          failed = true;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t dah = smem_desc_sw128(a_hi + s * C::kABytes);
          const uint64_t dbh = smem_desc_sw128(b_hi + s * L::kBBytes);
          uint64_t dal = 0, dbl = 0;
          if constexpr (C::kSplit) {
            dal = smem_desc_sw128(a_lo + s * C::kABytes);
            dbl = smem_desc_sw128(b_lo + s * L::kBBytes);
          }
          // bf16 tiles use the 64-byte swizzle: layout type 4 and 512-byte SBO.
          auto fix = [&](uint64_t d) -> uint64_t {
            if constexpr (PREC == kPrecBF16) {
              d &= ~(0x3FFFull << 32);
              d |= (uint64_t)(512u >> 4) << 32;
              d &= ~(7ull << 61);
              d |= 4ull << 61;
            }
            return d;
          };
#pragma unroll
          for (int kk = 0; kk < C::kKSteps; ++kk) {
            const uint64_t step = (uint64_t)(kk * C::kDescStep);
            const uint32_t acc = ((L::kPromote ? kin : kb) | kk) ? 1u : 0u;
            tc_mma<PREC == kPrecBF16 ? 1 : 0>(d_tmem, fix(dah + step), fix(dbh + step), idesc, acc);
            if constexpr (C::kSplit) {
              tc_mma<0>(d_tmem, dah + step, dbl + step, idesc, 1u);
              tc_mma<0>(d_tmem, dal + step, dbh + step, idesc, 1u);
            }
          }
          tc_commit(empty_bar(s));
          issued = true;
        }
        if constexpr (L::kPromote) {
          if (kin == L::kChunkKB - 1 || kb == p.num_kb - 1) {
            if (lane == 0) tc_commit(tfull_bar(cb));
            ++cc;
          }
        }
        __syncwarp();
      }
      if (failed) break;
      if constexpr (!L::kPromote) {
        if (lane == 0) tc_commit(tfull_bar(buf));
      }
      __syncwarp();
    }
    // Drain: every MMA issued by this thread has completed before TMEM is freed.
    if (lane == 0 && issued) {
      tc_commit(drain_bar);
      volatile int no_abort = 0;
      mbar_wait(drain_bar, 0, &no_abort, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int row_in_tile = warp * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    uint32_t cc = 0;
    for (int tj = 0; tj < my_tiles; ++tj) {
      int b, mt, nt;
      tile_coords(blockIdx.x + tj * gridDim.x, b, mt, nt);
      const int m = mt * kBM + row_in_tile;
      const bool row_ok = m < p.M;
      float* yrow = p.y + (long long)b * p.y_bstride + (long long)m * p.ldy;
      const float* rrow =
          p.res ? p.res + (long long)b * p.y_bstride + (long long)m * p.ldr : nullptr;
      if constexpr (L::kPromote) {
        // Fold each chunk accumulator into the running total (TMEM columns
        // [0, BN)) with round-to-nearest fp32 adds; the last chunk goes straight
        // to the output epilogue.
        const int nch = (p.num_kb + L::kChunkKB - 1) / L::kChunkKB;
        bool failed = false;
        for (int ch = 0; ch < nch; ++ch, ++cc) {
          const int cb = cc & 1;
          if (!mbar_wait(tfull_bar(cb), (cc >> 1) & 1, abort_flag, p.status)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const bool last = ch == nch - 1;
#pragma unroll 1
          for (int j = 0; j < BN / 32; ++j) {
            const int col0 = nt * BN + j * 32;
            if (col0 >= p.Nc) break;  // warp-uniform
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + lane_addr + BN * (1 + cb) + j * 32, r);
            if (ch > 0) {
              uint32_t t[32];
              tmem_ld_32x32b_x32(tmem_base + lane_addr + j * 32, t);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; ++e)
                r[e] = __float_as_uint(__uint_as_float(t[e]) + __uint_as_float(r[e]));
            } else {
              tmem_ld_wait();
            }
            if (!last)
              tmem_st_32x32b_x32(tmem_base + lane_addr + j * 32, r);
            else if (row_ok)
              store_row32(p, r, col0, yrow, rrow);
          }
          if (!last) tmem_st_wait();
          tc_fence_before();
          mbar_arrive(tempty_bar(cb));
        }
        if (failed) break;
      } else {
        const int buf = tj & 1;
        const uint32_t aph = (tj >> 1) & 1;
        if (!mbar_wait(tfull_bar(buf), aph, abort_flag, p.status)) break;
        tc_fence_after();
#pragma unroll 1
        for (int j = 0; j < BN / 32; ++j) {
          const int col0 = nt * BN + j * 32;
          if (col0 >= p.Nc) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + lane_addr + buf * BN + j * 32, r);
          tmem_ld_wait();
          if (row_ok) store_row32(p, r, col0, yrow, rrow);
        }
        tc_fence_before();
        mbar_arrive(tempty_bar(buf));
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

template <int PREC, int BN>
int launch_t(const IgemmParams& p, const CUtensorMap& hi, const CUtensorMap& lo, int num_sms,
             cudaStream_t st) {
  using L = Layout<PREC, BN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(igemm_tc_kernel<PREC, BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return (int)e;
    attr_set = true;
  }
  const int total = p.m_tiles * p.n_tiles * p.batches;
  const int grid = total < num_sms ? total : num_sms;
  if (grid <= 0) return 0;
  igemm_tc_kernel<PREC, BN><<<grid, kThreads, L::kBytes, st>>>(p, hi, lo);
  return (int)cudaGetLastError();
}

}  // namespace

int igemm_pick_bn(const IgemmParams& p, int precision, int num_sms) {
  const int nc = p.Nc;
  if (nc <= 64) return 64;
  // 3xTF32: the chunked accumulators (3 x BN) plus TMEM A slots must fit the
  // 512 TMEM columns; TF32 keeps only two whole-tile accumulators
  if (precision == kPrec3xTF32) return 128;
  const long long mt = (long long)((p.M + kBM - 1) / kBM) * p.batches;
  // Wide tiles halve A re-reads; use them when there are enough tiles to fill the GPU.
  if (nc >= 256 && mt * ((nc + 255) / 256) >= 2ll * num_sms) return 256;
  return 128;
}

int igemm_launch(const IgemmParams& p, const CUtensorMap& hi, const CUtensorMap& lo,
                 const CUtensorMap& am, int precision, int bn, int num_sms, cudaStream_t st) {
  if (p.a_mode != kALoadGather &&
      (precision == kPrecBF16 ||
       (p.a_mode == kALoadIm2colTaps ? ((p.Cs != 4 && p.Cs != 8 && p.Cs != 16) || p.K % p.Cs != 0)
        : p.a_mode == kALoadIm2col   ? p.Cs % 32 != 0
                                     : p.Cs < 32)))
    return (int)cudaErrorInvalidValue;
  // The kernel moves 16-byte vectors: refuse (instead of faulting on) any
  // pointer or stride that would make one of them misaligned.
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (!p.x || !p.y || mis(p.x) || mis(p.y) || (p.res && mis(p.res)) || (p.scale && mis(p.scale)) ||
      (p.shift && mis(p.shift)) || p.Cs % 4 || p.Nc % 4 || p.ldy % 4 || (p.res && p.ldr % 4) ||
      p.y_bstride % 4 || p.num_kb <= 0 || (p.batches > 1 && !p.a_off && p.M % 4))
    return (int)cudaErrorMisalignedAddress;
  if (precision == kPrec3xTF32 || precision == kPrecTF32)
    return igemm3_launch(p, hi, lo, am, precision, bn, num_sms, st);
#define OB2_CASE(PR, B)                                  \
  if (precision == PR && bn == B) return launch_t<PR, B>(p, hi, lo, num_sms, st);
  OB2_CASE(kPrecBF16, 64)
  OB2_CASE(kPrecBF16, 128)
  OB2_CASE(kPrecBF16, 256)
#undef OB2_CASE
  return (int)cudaErrorInvalidValue;
}

int pick_a_mode(const IgemmParams& p, int precision) {
  // A k-block is 32 fp32 (one 128-byte TMA row per pixel): 32 channels of one
  // filter tap, or 32 / Cs whole taps of a 4-, 8- or 16-channel tensor
  if (precision == kPrecBF16) return kALoadGather;
  const bool single_tap = p.K == p.Cs;
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
  if (p.a_mode == kALoadTma2d) {
    static EncodeTiledFn2 fn = reinterpret_cast<EncodeTiledFn2>(driver_fn("cuTensorMapEncodeTiled"));
    if (!fn) return (int)CUDA_ERROR_NOT_FOUND;
    // n = number of rows of the [rows][Cs] matrix (pixels of the batch, or all A rows)
    cuuint64_t dims[2] = {(cuuint64_t)p.Cs, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)p.Cs * 4};
    cuuint32_t box[2] = {32u, (cuuint32_t)kBM};
    cuuint32_t es[2] = {1u, 1u};
    return (int)fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  static EncodeIm2colFn fn = reinterpret_cast<EncodeIm2colFn>(driver_fn("cuTensorMapEncodeIm2col"));
  if (!fn) return (int)CUDA_ERROR_NOT_FOUND;
  // NHWC tensor, dims innermost first: C, W, H, N (n = images)
  cuuint64_t dims[4] = {(cuuint64_t)p.Cs, (cuuint64_t)p.Win, (cuuint64_t)p.Hin, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)p.Cs * 4, (cuuint64_t)p.Win * p.Cs * 4,
                           (cuuint64_t)p.Hin * p.Win * p.Cs * 4};
  // Bounding box of the base (top-left) input pixel of every output pixel:
  // W from -pw to (OW-1)*sw - pw, H likewise; traversal stride = conv stride.
  int lower[2] = {-p.pw, -p.ph};
  int upper[2] = {(p.OW - 1) * p.sw - p.pw - (p.Win - 1), (p.OH - 1) * p.sh - p.ph - (p.Hin - 1)};
  cuuint32_t es[4] = {1u, (cuuint32_t)p.sw, (cuuint32_t)p.sh, 1u};
  // taps mode: one box = all Cs channels (16 to 64 bytes) of 128 pixels for one
  // tap, unswizzled; otherwise 32 channels in 128-byte swizzled rows
  const bool taps = p.a_mode == kALoadIm2colTaps;
  return (int)fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, lower, upper,
                 taps ? (cuuint32_t)p.Cs : 32u, (cuuint32_t)kBM, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 taps ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace ob2
