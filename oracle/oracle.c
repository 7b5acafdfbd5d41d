/*
 * CPU oracle: plain-C restatement of the onnx-rs reference operators on the
 * Conv / MatMul / Gemm / MaxPool / GlobalAveragePool / Relu / Add path.
 *
 * TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline).  The product
 * library never links this file.  Each function cites the reference code it
 * restates (paths relative to the onnx-rs repository root).
 *
 * Threading mirrors the reference's rayon use: the batch dimension is split
 * across threads (conv.rs:882-934, conv.rs:1340-1365, matmul.rs:245-257).
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* threading helper                                                          */
/* ------------------------------------------------------------------------- */
typedef void (*orc_task_fn)(void* ctx, int64_t item);
typedef struct {
  orc_task_fn fn;
  void* ctx;
  int64_t begin, end;
} orc_range;

static void* orc_worker(void* p) {
  orc_range* r = (orc_range*)p;
  for (int64_t i = r->begin; i < r->end; ++i) r->fn(r->ctx, i);
  return NULL;
}

/* Runs fn(ctx, i) for i in [0, n) on up to nthreads threads, contiguous chunks. */
static void orc_parallel_for(int64_t n, int nthreads, orc_task_fn fn, void* ctx) {
  if (nthreads <= 1 || n <= 1) {
    for (int64_t i = 0; i < n; ++i) fn(ctx, i);
    return;
  }
  if (nthreads > n) nthreads = (int)n;
  pthread_t th[256];
  orc_range rg[256];
  if (nthreads > 256) nthreads = 256;
  int64_t chunk = (n + nthreads - 1) / nthreads;
  int started = 0;
  for (int t = 0; t < nthreads; ++t) {
    rg[t].fn = fn;
    rg[t].ctx = ctx;
    rg[t].begin = t * chunk;
    rg[t].end = (t + 1) * chunk < n ? (t + 1) * chunk : n;
    if (rg[t].begin >= rg[t].end) break;
    if (pthread_create(&th[t], NULL, orc_worker, &rg[t]) != 0) {
      orc_worker(&rg[t]); /* run inline if a thread cannot be created */
      rg[t].begin = rg[t].end;
      th[t] = 0;
    }
    started = t + 1;
  }
  for (int t = 0; t < started; ++t)
    if (th[t]) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------- */
/* shapes and strategy                                                       */
/* ------------------------------------------------------------------------- */
/* conv.rs:317-320: out = (in + pad_head + pad_tail - ((k-1)*d + 1)) / s + 1 */
int64_t orc_conv_out_dim(int64_t in, int64_t k, int64_t stride, int64_t pad_head,
                         int64_t pad_tail, int64_t dilation) {
  int64_t dk = (k - 1) * dilation + 1;
  int64_t span = in + pad_head + pad_tail - dk;
  if (span < 0 || stride <= 0) return 0;
  return span / stride + 1;
}

/* conv.rs:426-458 */
void orc_same_pads(int64_t in, int64_t k, int64_t stride, int64_t dilation, int mode,
                   int64_t* pad_head, int64_t* pad_tail) {
  int64_t dk = (k - 1) * dilation + 1;
  int64_t out = (in + stride - 1) / stride;
  int64_t need = (out - 1) * stride + dk - in;
  *pad_head = 0;
  *pad_tail = 0;
  if (need > 0) {
    if (mode == 1) { /* SAME_UPPER */
      *pad_head = need / 2;
      *pad_tail = need - *pad_head;
    } else { /* SAME_LOWER */
      *pad_tail = need / 2;
      *pad_head = need - *pad_tail;
    }
  }
}

/* conv.rs:1425-1452 (2-D branch of optimize_convolution_strategy) */
int orc_conv_strategy(int64_t kh, int64_t kw, int64_t group) {
  int p2h = (kh == 1 || kh == 2 || kh == 4 || kh == 8);
  int p2w = (kw == 1 || kw == 2 || kw == 4 || kw == 8);
  if (p2h && p2w && group == 1) return ORC_CONV_SIMD;
  if (kh <= 5 && kw <= 5 && group <= 4) return ORC_CONV_IM2COL;
  if (kh > 11 || kw > 11) return ORC_CONV_DIRECT;
  return ORC_CONV_IM2COL;
}

/* ------------------------------------------------------------------------- */
/* plain fp32 GEMM used where the reference calls ndarray general_mat_mul     */
/* C[m][n] = sum_k A[m][k] * B[k][n], summed in k order (i-k-j loop).          */
/* ------------------------------------------------------------------------- */
#define ORC_JB 512
__attribute__((optimize("fp-contract=fast")))
static void orc_sgemm_f32(const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
                          int64_t ldc, int64_t M, int64_t N, int64_t K) {
  for (int64_t j0 = 0; j0 < N; j0 += ORC_JB) {
    int64_t jn = N - j0 < ORC_JB ? N - j0 : ORC_JB;
    for (int64_t i = 0; i < M; ++i) {
      float* c = C + i * ldc + j0;
      for (int64_t j = 0; j < jn; ++j) c[j] = 0.0f;
      const float* a = A + i * lda;
      for (int64_t p = 0; p < K; ++p) {
        const float av = a[p];
        const float* b = B + p * ldb + j0;
        for (int64_t j = 0; j < jn; ++j) c[j] += av * b[j];
      }
    }
  }
}

static void orc_sgemm_f64acc(const float* A, int64_t lda, const float* B, int64_t ldb,
                             float* C, int64_t ldc, int64_t M, int64_t N, int64_t K) {
  double acc[ORC_JB];
  for (int64_t j0 = 0; j0 < N; j0 += ORC_JB) {
    int64_t jn = N - j0 < ORC_JB ? N - j0 : ORC_JB;
    for (int64_t i = 0; i < M; ++i) {
      for (int64_t j = 0; j < jn; ++j) acc[j] = 0.0;
      const float* a = A + i * lda;
      for (int64_t p = 0; p < K; ++p) {
        const double av = a[p];
        const float* b = B + p * ldb + j0;
        for (int64_t j = 0; j < jn; ++j) acc[j] += av * (double)b[j];
      }
      float* c = C + i * ldc + j0;
      for (int64_t j = 0; j < jn; ++j) c[j] = (float)acc[j];
    }
  }
}

static void orc_sgemm(int acc64, const float* A, int64_t lda, const float* B, int64_t ldb,
                      float* C, int64_t ldc, int64_t M, int64_t N, int64_t K) {
  if (acc64)
    orc_sgemm_f64acc(A, lda, B, ldb, C, ldc, M, N, K);
  else
    orc_sgemm_f32(A, lda, B, ldb, C, ldc, M, N, K);
}

/* ------------------------------------------------------------------------- */
/* Conv 2-D                                                                  */
/* ------------------------------------------------------------------------- */
typedef struct {
  const float *x, *w, *bias;
  float* y;
  int64_t c, h, wd, co, kh, kw, oh, ow;
  int64_t sh, sw, pt, pl, dh, dw, group;
  int acc64, simd;
} orc_conv_ctx;

/* compute_conv2d_direct_impl (conv.rs:849-935); `simd` adds the +0.0 that
 * compute_conv_simd applies afterwards (conv.rs:757-768). */
/* Every output element is the fp32 sum over (ic, kh, kw) in that order, as in
 * the reference's loop nest; the loops are interchanged so that the innermost
 * loop runs over output columns (one accumulator plane per output channel),
 * which leaves each element's summation order -- and so its value -- unchanged. */
static void orc_conv_direct_batch(void* p, int64_t b) {
  const orc_conv_ctx* k = (const orc_conv_ctx*)p;
  const int64_t cg = k->c / k->group, cog = k->co / k->group;
  const int64_t plane = k->oh * k->ow;
  float* acc = (float*)malloc((size_t)plane * sizeof(float));
  double* accd = k->acc64 ? (double*)malloc((size_t)plane * sizeof(double)) : NULL;
  if (!acc || (k->acc64 && !accd)) {
    free(acc);
    free(accd);
    return;
  }
  for (int64_t g = 0; g < k->group; ++g) {
    for (int64_t oc = g * cog; oc < (g + 1) * cog; ++oc) {
      const float* wo = k->w + oc * cg * k->kh * k->kw;
      for (int64_t i = 0; i < plane; ++i) acc[i] = 0.0f;
      if (accd)
        for (int64_t i = 0; i < plane; ++i) accd[i] = 0.0;
      for (int64_t ic = g * cg; ic < (g + 1) * cg; ++ic) {
        const int64_t icg = ic - g * cg;
        const float* xp = k->x + (b * k->c + ic) * k->h * k->wd;
        for (int64_t r = 0; r < k->kh; ++r) {
          for (int64_t s = 0; s < k->kw; ++s) {
            const float wv = wo[(icg * k->kh + r) * k->kw + s];
            /* output columns whose input column is in bounds */
            const int64_t off = s * k->dw - k->pl;
            int64_t ow0 = off >= 0 ? 0 : (-off + k->sw - 1) / k->sw;
            int64_t ow1 = k->wd - 1 - off < 0 ? -1 : (k->wd - 1 - off) / k->sw;
            if (ow1 > k->ow - 1) ow1 = k->ow - 1;
            for (int64_t oh = 0; oh < k->oh; ++oh) {
              const int64_t ih = oh * k->sh - k->pt + r * k->dh;
              if (ih < 0 || ih >= k->h) continue;
              const float* xr = xp + ih * k->wd + off;
              float* ar = acc + oh * k->ow;
              if (accd) {
                double* dr = accd + oh * k->ow;
                for (int64_t ow = ow0; ow <= ow1; ++ow) dr[ow] += (double)xr[ow * k->sw] * (double)wv;
              } else if (k->sw == 1) {
                for (int64_t ow = ow0; ow <= ow1; ++ow) ar[ow] += xr[ow] * wv;
              } else {
                for (int64_t ow = ow0; ow <= ow1; ++ow) ar[ow] += xr[ow * k->sw] * wv;
              }
            }
          }
        }
      }
      float* yo = k->y + (b * k->co + oc) * plane;
      for (int64_t i = 0; i < plane; ++i) {
        float sum = accd ? (float)accd[i] : acc[i];
        if (k->bias) sum += k->bias[oc];
        if (k->simd) sum += 0.0f;
        yo[i] = sum;
      }
    }
  }
  free(acc);
  free(accd);
}

/* compute_conv2d_im2col (conv.rs:1142-1261) with im2col_2d (conv.rs:1309-1368):
 * build the [C, kh, kw, OH*OW] column buffer of one image, multiply each group's
 * [CO/g, C/g*kh*kw] weight matrix with it, then add the bias. */
static void orc_conv_im2col_batch(void* p, int64_t b) {
  const orc_conv_ctx* k = (const orc_conv_ctx*)p;
  const int64_t ohw = k->oh * k->ow;
  const int64_t rows = k->c * k->kh * k->kw;
  float* col = (float*)malloc((size_t)(rows * ohw) * sizeof(float));
  if (!col) return;
  for (int64_t c = 0; c < k->c; ++c) {
    const float* xp = k->x + (b * k->c + c) * k->h * k->wd;
    for (int64_t r = 0; r < k->kh; ++r)
      for (int64_t s = 0; s < k->kw; ++s) {
        float* cp = col + ((c * k->kh + r) * k->kw + s) * ohw;
        for (int64_t oh = 0; oh < k->oh; ++oh)
          for (int64_t ow = 0; ow < k->ow; ++ow) {
            int64_t ih = oh * k->sh - k->pt + r * k->dh;
            int64_t iw = ow * k->sw - k->pl + s * k->dw;
            cp[oh * k->ow + ow] =
                (ih >= 0 && ih < k->h && iw >= 0 && iw < k->wd) ? xp[ih * k->wd + iw] : 0.0f;
          }
      }
  }
  const int64_t cg = k->c / k->group, cog = k->co / k->group;
  const int64_t kg = cg * k->kh * k->kw;
  for (int64_t g = 0; g < k->group; ++g) {
    const float* wg = k->w + g * cog * kg;
    const float* cgp = col + g * kg * ohw;
    float* yg = k->y + (b * k->co + g * cog) * ohw;
    orc_sgemm(k->acc64, wg, kg, cgp, ohw, yg, ohw, cog, ohw, kg);
    if (k->bias)
      for (int64_t o = 0; o < cog; ++o) {
        const float bv = k->bias[g * cog + o];
        float* yr = yg + o * ohw;
        for (int64_t i = 0; i < ohw; ++i) yr[i] += bv;
      }
  }
  free(col);
}

int orc_conv2d(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, const float* wt,
               int64_t co, int64_t kh, int64_t kw, const float* bias, int64_t sh, int64_t sw,
               int64_t pt, int64_t pl, int64_t pb, int64_t pr, int64_t dh, int64_t dw,
               int64_t group, int strategy, int acc64, int nthreads, float* y) {
  /* validation as compute_conv_direct (conv.rs:628-644) */
  if (group <= 0 || c % group != 0 || co % group != 0) return ORC_ERR_VALIDATION;
  if (sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0) return ORC_ERR_VALIDATION;
  orc_conv_ctx k;
  k.x = x;
  k.w = wt;
  k.bias = bias;
  k.y = y;
  k.c = c;
  k.h = h;
  k.wd = w;
  k.co = co;
  k.kh = kh;
  k.kw = kw;
  k.oh = orc_conv_out_dim(h, kh, sh, pt, pb, dh);
  k.ow = orc_conv_out_dim(w, kw, sw, pl, pr, dw);
  k.sh = sh;
  k.sw = sw;
  k.pt = pt;
  k.pl = pl;
  k.dh = dh;
  k.dw = dw;
  k.group = group;
  k.acc64 = acc64;
  k.simd = 0;
  if (strategy == ORC_CONV_AUTO) strategy = orc_conv_strategy(kh, kw, group);
  if (strategy == ORC_CONV_IM2COL)
    orc_parallel_for(n, nthreads, orc_conv_im2col_batch, &k);
  else {
    k.simd = (strategy == ORC_CONV_SIMD);
    orc_parallel_for(n, nthreads, orc_conv_direct_batch, &k);
  }
  return ORC_OK;
}

/* compute_conv_direct for 1-D / 2-D / 3-D (conv.rs:609-706 and the per-rank
 * direct impls): loops over (oc, output position, ic, kernel taps). */
int orc_conv_nd_direct(const float* x, const int64_t* xs, int rank, const float* wt,
                       const int64_t* ws, const float* bias, const int64_t* strides,
                       const int64_t* pads, const int64_t* dil, int64_t group, float* y,
                       int64_t* ys) {
  if (rank < 3 || rank > 5) return ORC_ERR_VALIDATION;
  const int sd = rank - 2;
  const int64_t n = xs[0], c = xs[1], co = ws[0];
  if (group <= 0 || c % group || co % group || ws[1] != c / group) return ORC_ERR_VALIDATION;
  int64_t in[3] = {1, 1, 1}, kk[3] = {1, 1, 1}, out[3] = {1, 1, 1};
  int64_t st[3] = {1, 1, 1}, dl[3] = {1, 1, 1}, ph[3] = {0, 0, 0};
  for (int i = 0; i < sd; ++i) {
    in[i] = xs[i + 2];
    kk[i] = ws[i + 2];
    st[i] = strides[i];
    dl[i] = dil[i];
    ph[i] = pads[i];
    out[i] = orc_conv_out_dim(in[i], kk[i], st[i], pads[i], pads[i + sd], dl[i]);
  }
  ys[0] = n;
  ys[1] = co;
  for (int i = 0; i < sd; ++i) ys[i + 2] = out[i];
  const int64_t cg = c / group, cog = co / group;
  for (int64_t b = 0; b < n; ++b)
    for (int64_t oc = 0; oc < co; ++oc) {
      const int64_t g = oc / cog;
      for (int64_t o0 = 0; o0 < out[0]; ++o0)
        for (int64_t o1 = 0; o1 < out[1]; ++o1)
          for (int64_t o2 = 0; o2 < out[2]; ++o2) {
            float sum = 0.0f;
            for (int64_t icg = 0; icg < cg; ++icg) {
              const int64_t ic = g * cg + icg;
              for (int64_t k0 = 0; k0 < kk[0]; ++k0)
                for (int64_t k1 = 0; k1 < kk[1]; ++k1)
                  for (int64_t k2 = 0; k2 < kk[2]; ++k2) {
                    int64_t i0 = o0 * st[0] - ph[0] + k0 * dl[0];
                    int64_t i1 = o1 * st[1] - ph[1] + k1 * dl[1];
                    int64_t i2 = o2 * st[2] - ph[2] + k2 * dl[2];
                    if (i0 < 0 || i0 >= in[0] || i1 < 0 || i1 >= in[1] || i2 < 0 || i2 >= in[2])
                      continue;
                    float xv = x[(((b * c + ic) * in[0] + i0) * in[1] + i1) * in[2] + i2];
                    float wv = wt[(((oc * cg + icg) * kk[0] + k0) * kk[1] + k1) * kk[2] + k2];
                    sum += xv * wv;
                  }
            }
            if (bias) sum += bias[oc];
            y[(((b * co + oc) * out[0] + o0) * out[1] + o1) * out[2] + o2] = sum;
          }
    }
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* MatMul                                                                    */
/* ------------------------------------------------------------------------- */
/* broadcast_batch_dims (matmul.rs:497-546): right-aligned, 1 broadcasts. */
static int orc_bcast_batch(const int64_t* a, int ra, const int64_t* b, int rb, int64_t* out,
                           int* ro) {
  int r = ra > rb ? ra : rb;
  for (int i = 0; i < r; ++i) {
    int64_t da = i >= r - ra ? a[i - (r - ra)] : 1;
    int64_t db = i >= r - rb ? b[i - (r - rb)] : 1;
    if (da == 1)
      out[i] = db;
    else if (db == 1 || da == db)
      out[i] = da;
    else
      return ORC_ERR_VALIDATION;
  }
  *ro = r;
  return ORC_OK;
}

/* validate_matmul_shapes (matmul.rs:401-487) */
int orc_matmul_shape(const int64_t* as, int ra, const int64_t* bs, int rb, int64_t* out,
                     int* ro) {
  if (ra == 0 || rb == 0) return ORC_ERR_VALIDATION;
  if (ra == 1 && rb == 1) {
    if (as[0] != bs[0]) return ORC_ERR_VALIDATION;
    *ro = 0;
    return ORC_OK;
  }
  if (ra == 1) {
    if (as[0] != bs[rb - 2]) return ORC_ERR_VALIDATION;
    for (int i = 0; i < rb - 2; ++i) out[i] = bs[i];
    out[rb - 2] = bs[rb - 1];
    *ro = rb - 1;
    return ORC_OK;
  }
  if (rb == 1) {
    if (as[ra - 1] != bs[0]) return ORC_ERR_VALIDATION;
    for (int i = 0; i < ra - 2; ++i) out[i] = as[i];
    out[ra - 2] = as[ra - 2];
    *ro = ra - 1;
    return ORC_OK;
  }
  if (as[ra - 1] != bs[rb - 2]) return ORC_ERR_VALIDATION;
  int r = 0;
  if (ra > 2 || rb > 2) {
    if (orc_bcast_batch(as, ra - 2, bs, rb - 2, out, &r) != ORC_OK) return ORC_ERR_VALIDATION;
  }
  out[r] = as[ra - 2];
  out[r + 1] = bs[rb - 1];
  *ro = r + 2;
  return ORC_OK;
}

/* create_broadcast_indices (matmul.rs:587-643): flat input batch index of
 * output batch `o` for an input whose batch dims are `in` (right-aligned). */
static int64_t orc_bcast_index(int64_t o, const int64_t* outd, int ro, const int64_t* in,
                               int ri) {
  int64_t idx = 0, stride = 1, rem = o;
  for (int i = ro - 1; i >= 0; --i) {
    int64_t d = outd[i];
    if (d == 0) continue;
    int64_t coord = rem % d;
    rem /= d;
    int j = i - (ro - ri);
    if (j >= 0) {
      if (in[j] != 1) idx += coord * stride;
      stride *= in[j];
    }
  }
  return idx;
}

typedef struct {
  const float *a, *b;
  float* y;
  int64_t m, n, k;
  int64_t bat_out[8];
  int ro;
  int64_t ba[8], bb[8];
  int rba, rbb;
  int acc64;
} orc_mm_ctx;

static void orc_mm_batch(void* p, int64_t i) {
  const orc_mm_ctx* c = (const orc_mm_ctx*)p;
  int64_t ia = orc_bcast_index(i, c->bat_out, c->ro, c->ba, c->rba);
  int64_t ib = orc_bcast_index(i, c->bat_out, c->ro, c->bb, c->rbb);
  orc_sgemm(c->acc64, c->a + ia * c->m * c->k, c->k, c->b + ib * c->k * c->n, c->n,
            c->y + i * c->m * c->n, c->n, c->m, c->n, c->k);
}

/* compute_matmul (matmul.rs:124-279) incl. compute_vector_matmul (:282-398):
 * 1-D operands are promoted (prepend / append a 1) and the added dim removed. */
int orc_matmul(const float* a, const int64_t* as, int ra, const float* b, const int64_t* bs,
               int rb, int acc64, int nthreads, float* y) {
  int64_t outs[10];
  int ro;
  if (ra > 8 || rb > 8) return ORC_ERR_UNSUPPORTED;
  if (orc_matmul_shape(as, ra, bs, rb, outs, &ro) != ORC_OK) return ORC_ERR_VALIDATION;
  int64_t a2[10], b2[10];
  int ra2 = ra, rb2 = rb;
  if (ra == 1) {
    a2[0] = 1;
    a2[1] = as[0];
    ra2 = 2;
  } else
    memcpy(a2, as, sizeof(int64_t) * ra);
  if (rb == 1) {
    b2[0] = bs[0];
    b2[1] = 1;
    rb2 = 2;
  } else
    memcpy(b2, bs, sizeof(int64_t) * rb);
  orc_mm_ctx c;
  c.a = a;
  c.b = b;
  c.y = y;
  c.m = a2[ra2 - 2];
  c.k = a2[ra2 - 1];
  c.n = b2[rb2 - 1];
  c.acc64 = acc64;
  c.rba = ra2 - 2;
  c.rbb = rb2 - 2;
  memcpy(c.ba, a2, sizeof(int64_t) * c.rba);
  memcpy(c.bb, b2, sizeof(int64_t) * c.rbb);
  c.ro = 0;
  if (c.rba > 0 || c.rbb > 0) orc_bcast_batch(c.ba, c.rba, c.bb, c.rbb, c.bat_out, &c.ro);
  int64_t nb = 1;
  for (int i = 0; i < c.ro; ++i) nb *= c.bat_out[i];
  /* matmul.rs:191,244: parallel only for more than 8 output batches */
  orc_parallel_for(nb, nb > 8 ? nthreads : 1, orc_mm_batch, &c);
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* Gemm (ONNX semantics; the reference's compute_gemm, gemm.rs:172-291)      */
/* ------------------------------------------------------------------------- */
int orc_gemm(const float* a, const float* b, const float* c, const int64_t* cs, int c_rank,
             int64_t m, int64_t nn, int64_t k, int trans_a, int trans_b, float alpha,
             float beta, int acc64, float* y) {
  int64_t cm = 1, cn = 1;
  if (c) {
    if (c_rank == 1) {
      cn = cs[0];
    } else if (c_rank == 2) {
      cm = cs[0];
      cn = cs[1];
    } else if (c_rank != 0)
      return ORC_ERR_VALIDATION;
    if ((cm != 1 && cm != m) || (cn != 1 && cn != nn)) return ORC_ERR_VALIDATION;
  }
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < nn; ++j) {
      float s = 0.0f;
      double sd = 0.0;
      for (int64_t p = 0; p < k; ++p) {
        float av = trans_a ? a[p * m + i] : a[i * k + p];
        float bv = trans_b ? b[j * k + p] : b[p * nn + j];
        if (acc64)
          sd += (double)av * (double)bv;
        else
          s += av * bv;
      }
      if (acc64) s = (float)sd;
      float v = alpha * s;
      if (c && beta != 0.0f) {
        int64_t ci = (cm == 1 ? 0 : i) * cn + (cn == 1 ? 0 : j);
        v += beta * c[ci];
      }
      y[i * nn + j] = v;
    }
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* Pooling                                                                   */
/* ------------------------------------------------------------------------- */
/* max_pool (pool.rs:307-393): init f32::MIN, in-bounds taps only, f32::max
 * (which ignores a NaN operand).  Output size floor mode (pool.rs:343-344);
 * ceil_mode follows the planner's infer_pool_shape (planner.rs:1230). */
int orc_maxpool2d(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int64_t kh,
                  int64_t kw, int64_t sh, int64_t sw, int64_t pt, int64_t pl, int64_t pb,
                  int64_t pr, int ceil_mode, float* y, int64_t* indices) {
  if (sh <= 0 || sw <= 0 || kh <= 0 || kw <= 0) return ORC_ERR_VALIDATION;
  int64_t oh, ow;
  if (ceil_mode) {
    oh = (h + pt + pb - kh + sh - 1) / sh + 1;
    ow = (w + pl + pr - kw + sw - 1) / sw + 1;
  } else {
    oh = (h + pt + pb - kh) / sh + 1;
    ow = (w + pl + pr - kw) / sw + 1;
  }
  for (int64_t b = 0; b < n; ++b)
    for (int64_t ch = 0; ch < c; ++ch)
      for (int64_t i = 0; i < oh; ++i)
        for (int64_t j = 0; j < ow; ++j) {
          float mv = -3.40282347e+38f; /* f32::MIN */
          int64_t mi = -1;
          for (int64_t r = 0; r < kh; ++r)
            for (int64_t s = 0; s < kw; ++s) {
              int64_t ih = i * sh - pt + r, iw = j * sw - pl + s;
              if (ih >= 0 && ih < h && iw >= 0 && iw < w) {
                int64_t xi = ((b * c + ch) * h + ih) * w + iw;
                float v = x[xi];
                if (v > mv || (mi < 0 && v == mv)) {
                  mv = v;
                  mi = xi;
                }
              }
            }
          int64_t yi = ((b * c + ch) * oh + i) * ow + j;
          y[yi] = mv;
          if (indices) indices[yi] = mi;
        }
  return ORC_OK;
}

/* global_pool GlobalAverage (pool.rs:493-557): sum in fp32 in scan order,
 * then sum / count as f32. */
int orc_global_avgpool(const float* x, int64_t n, int64_t c, int64_t spatial, float* y) {
  for (int64_t i = 0; i < n * c; ++i) {
    float s = 0.0f;
    const float* p = x + i * spatial;
    for (int64_t j = 0; j < spatial; ++j) s += p[j];
    y[i] = spatial > 0 ? s / (float)spatial : 0.0f;
  }
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* Elementwise                                                               */
/* ------------------------------------------------------------------------- */
void orc_relu(const float* x, int64_t count, float* y) {
  for (int64_t i = 0; i < count; ++i) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* get_broadcast_shape (tensor.rs:1536-1571) */
int orc_broadcast_shape(const int64_t* as, int ra, const int64_t* bs, int rb, int64_t* out,
                        int* ro) {
  return orc_bcast_batch(as, ra, bs, rb, out, ro);
}

/* element_wise_binary_op with op = a + b (tensor.rs:1124-1218): both operands
 * broadcast to the common shape (broadcast_to, tensor.rs:993-1080). */
int orc_add(const float* a, const int64_t* as, int ra, const float* b, const int64_t* bs,
            int rb, float* y) {
  int64_t out[16];
  int ro;
  if (ra > 16 || rb > 16) return ORC_ERR_UNSUPPORTED;
  if (orc_bcast_batch(as, ra, bs, rb, out, &ro) != ORC_OK) return ORC_ERR_VALIDATION;
  int64_t total = 1;
  for (int i = 0; i < ro; ++i) total *= out[i];
  for (int64_t o = 0; o < total; ++o) {
    int64_t ia = orc_bcast_index(o, out, ro, as, ra);
    int64_t ib = orc_bcast_index(o, out, ro, bs, rb);
    y[o] = a[ia] + b[ib];
  }
  return ORC_OK;
}

/* ONNX BatchNormalization, inference mode (no reference operator exists). */
int orc_batchnorm(const float* x, int64_t n, int64_t c, int64_t spatial, const float* scale,
                  const float* bias, const float* mean, const float* var, float eps, float* y) {
  for (int64_t b = 0; b < n; ++b)
    for (int64_t ch = 0; ch < c; ++ch) {
      const float den = sqrtf(var[ch] + eps);
      const float* xp = x + (b * c + ch) * spatial;
      float* yp = y + (b * c + ch) * spatial;
      for (int64_t j = 0; j < spatial; ++j) yp[j] = (xp[j] - mean[ch]) / den * scale[ch] + bias[ch];
    }
  return ORC_OK;
}
