/*
 * b2m_oracle.c — CPU restatement of the reference's MatMul-family arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA kernels in
 * onnx_runtime_dart_b200/csrc are compared against; it is also the timed CPU
 * baseline of bench.py. Nothing in the product library links or calls it.
 *
 * What it restates (reference = onnx_runtime_dart, pure Dart):
 *   - matmulKernel            lib/src/gemm_kernel_simd.dart:32-243 (+ _gemv :459-614,
 *                             _matmulSmallM :616-677, _matmul4x16Direct :244-389)
 *   - opMatMul                lib/src/onnx_ops.dart:1710-1766
 *   - opGemm                  lib/src/onnx_ops.dart:2152-2173
 *   - opMatMulInteger         lib/src/onnx_qlinear_ops.dart:32-81
 *   - opQLinearMatMul         lib/src/onnx_qlinear_ops.dart:85-108 (+ _roundEven :19-26)
 *   - opMatMulNBits           lib/src/onnx_qlinear_ops.dart:115-228
 *   - opConv (im2col, depthwise, 3-D and the Winograd F(2x2,3x3) branch),
 *     ConvInteger / QLinearConv, ConvTranspose, DynamicQuantizeLinear
 *
 * Numerics. Dart's Float32x4 lanes multiply and add with separate float32
 * rounding (SSE mulps/addps, no FMA), and scalar Dart `double` code rounds in
 * binary64 and only narrows to float32 on a Float32List store. This file is
 * compiled with -O2 -ffp-contract=off -fno-fast-math on x86-64 (SSE math,
 * FLT_EVAL_METHOD 0), so `float` expressions here round exactly like a
 * Float32x4 lane and `double` expressions like a Dart double.
 *
 * Parallelism. The reference's only parallel strategy is the isolate pool's
 * output-column split (lib/src/parallel_pool.dart:236-260); every column is
 * computed by exactly the same sequence of operations whichever worker owns
 * it, so results are bitwise independent of `nthreads`. The same split is
 * used here (pthreads) so the CPU baseline can use all host cores.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* fp32 GEMM: matmulKernel                                                    */
/* ------------------------------------------------------------------------- */

/*
 * One output column j of out[m x n] = a[m x k] . b[k x n] (row-major).
 *
 * Which accumulator the reference uses for a column depends only on (m, n, j):
 *   m >= 4          every column is a Float32x4 lane (4x16 direct tile :244,
 *                   narrow tile :391 or packed 4x8 panel with zero-filled tail
 *                   lanes :100-242) -> float acc, k order.
 *   m == 1 / m < 4  columns below n & ~3 are Float32x4 lanes (_gemvAligned
 *                   :480, _gemvScalar :543-600, _matmulSmallM :616-663);
 *                   the n % 4 tail columns use a `double` accumulator
 *                   (_gemvScalar :601-608, _matmulSmallM :665-672).
 * Panel / tile widths never change the k order (the file comment at :12-15
 * and the pool's bitwise-equality contract rely on this), so one column can be
 * produced independently of its neighbours.
 */
static void gemm_column(const float *a, int64_t lda, const float *b, int64_t ldb,
                        float *out, int64_t ldo, int64_t m, int64_t k, int64_t n,
                        int64_t j) {
  const int double_tail = (m < 4) && (j >= (n & ~(int64_t)3));
  for (int64_t i = 0; i < m; i++) {
    const float *ar = a + i * lda;
    if (double_tail) {
      double acc = 0.0;
      for (int64_t kk = 0; kk < k; kk++) acc += (double)ar[kk] * (double)b[kk * ldb + j];
      out[i * ldo + j] = (float)acc;
    } else {
      float acc = 0.0f;
      for (int64_t kk = 0; kk < k; kk++) {
        const float p = ar[kk] * b[kk * ldb + j];
        acc = acc + p;
      }
      out[i * ldo + j] = acc;
    }
  }
}

typedef struct {
  const float *a;
  const float *b;
  float *out;
  int64_t m, k, n, ldo, j0, j1;
} gemm_job;

static void *gemm_worker(void *p) {
  gemm_job *g = (gemm_job *)p;
  for (int64_t j = g->j0; j < g->j1; j++)
    gemm_column(g->a, g->k, g->b, g->n, g->out, g->ldo, g->m, g->k, g->n, j);
  return NULL;
}

/* Column slices per worker: the pool's split (parallel_pool.dart:236-239). */
static void run_column_split(void *(*fn)(void *), void *jobs, size_t job_size, int64_t n,
                             int nthreads, void (*set_range)(void *, int64_t, int64_t)) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > n) nthreads = (int)(n > 0 ? n : 1);
  pthread_t tid[256];
  if (nthreads > 256) nthreads = 256;
  int64_t base = n / nthreads, rem = n % nthreads, start = 0;
  for (int t = 0; t < nthreads; t++) {
    int64_t cnt = base + (t < rem ? 1 : 0);
    void *job = (char *)jobs + (size_t)t * job_size;
    set_range(job, start, start + cnt);
    start += cnt;
  }
  if (nthreads == 1) {
    fn(jobs);
    return;
  }
  for (int t = 0; t < nthreads; t++) pthread_create(&tid[t], NULL, fn, (char *)jobs + (size_t)t * job_size);
  for (int t = 0; t < nthreads; t++) pthread_join(tid[t], NULL);
}

static void gemm_set_range(void *p, int64_t j0, int64_t j1) {
  ((gemm_job *)p)->j0 = j0;
  ((gemm_job *)p)->j1 = j1;
}

/* matmulKernel(a, aOff, b, bOff, out, outOff, m, k, n, outStride: ldo). */
ORC_API void orc_matmul_kernel(const float *a, const float *b, float *out, int64_t m, int64_t k,
                               int64_t n, int64_t ldo, int nthreads) {
  gemm_job jobs[256];
  for (int t = 0; t < 256; t++) {
    jobs[t].a = a;
    jobs[t].b = b;
    jobs[t].out = out;
    jobs[t].m = m;
    jobs[t].k = k;
    jobs[t].n = n;
    jobs[t].ldo = ldo;
  }
  run_column_split(gemm_worker, jobs, sizeof(gemm_job), n, nthreads, gemm_set_range);
}

/* ------------------------------------------------------------------------- */
/* opMatMul: numpy-broadcast batches (onnx_ops.dart:1710-1766)                */
/* ------------------------------------------------------------------------- */

/* _flattenBroadcast (onnx_ops.dart:57-70): flat batch index of src for the
 * output batch coordinates (leading dims of size 1 broadcast). */
static int64_t flatten_broadcast(const int64_t *out_coords, int out_rank, const int64_t *src,
                                 int src_rank) {
  int64_t flat = 0, stride = 1;
  for (int d = src_rank - 1; d >= 0; d--) {
    int od = d + (out_rank - src_rank);
    int64_t coord = src[d] == 1 ? 0 : out_coords[od];
    flat += coord * stride;
    stride *= src[d];
  }
  return flat;
}

/* Returns 0 on success, -1 if the batch shapes do not broadcast. */
ORC_API int orc_matmul(const float *a, const int64_t *a_shape, int a_rank, const float *b,
                       const int64_t *b_shape, int b_rank, float *out, int nthreads) {
  if (a_rank < 2 || b_rank < 2 || a_rank > 16 || b_rank > 16) return -1;
  const int64_t m = a_shape[a_rank - 2], k = a_shape[a_rank - 1];
  const int64_t n = b_shape[b_rank - 1];
  if (b_shape[b_rank - 2] != k) return -1;
  const int ab = a_rank - 2, bb = b_rank - 2;
  const int rank = ab > bb ? ab : bb;
  int64_t out_batch[16], ap[16], bp[16];
  for (int d = 0; d < rank; d++) {
    ap[d] = d < rank - ab ? 1 : a_shape[d - (rank - ab)];
    bp[d] = d < rank - bb ? 1 : b_shape[d - (rank - bb)];
    if (ap[d] == bp[d]) out_batch[d] = ap[d];
    else if (ap[d] == 1) out_batch[d] = bp[d];
    else if (bp[d] == 1) out_batch[d] = ap[d];
    else return -1;
  }
  int64_t batch_count = 1, b_count = 1;
  for (int d = 0; d < rank; d++) batch_count *= out_batch[d];
  for (int d = 0; d < bb; d++) b_count *= b_shape[d];
  if (batch_count * m * n > 0) memset(out, 0, sizeof(float) * (size_t)(batch_count * m * n));
  /* Shared 2-D B: collapse every batch of A into one GEMM (:1728-1735). This
   * changes m (and so the kernel variant) and is part of the numerics. */
  if (batch_count > 1 && b_count == 1) {
    orc_matmul_kernel(a, b, out, batch_count * m, k, n, n, nthreads);
    return 0;
  }
  int64_t coords[16];
  for (int64_t batch = 0; batch < batch_count; batch++) {
    int64_t rem = batch;
    for (int d = rank - 1; d >= 0; d--) {
      int64_t dim = out_batch[d] == 0 ? 1 : out_batch[d];
      coords[d] = rem % dim;
      rem /= dim;
    }
    int64_t af = flatten_broadcast(coords, rank, a_shape, ab);
    int64_t bf = flatten_broadcast(coords, rank, b_shape, bb);
    orc_matmul_kernel(a + af * m * k, b + bf * k * n, out + batch * m * n, m, k, n, n, nthreads);
  }
  return 0;
}

/* ------------------------------------------------------------------------- */
/* opGemm (onnx_ops.dart:2152-2173; prepack onnx_graph.dart:2156-2161)        */
/* ------------------------------------------------------------------------- */

/*
 * y[M x N] = alpha * A' . B' + beta * C, A' = transA ? A^T : A (A stored
 * [K x M] when transposed), B' likewise. The transposes are plain copies
 * (opTranspose), the product goes through opMatMul (2-D, no batches), alpha
 * multiplies in place only when != 1 (:2164-2168), beta scales C only when
 * != 1 (:2170), and the add is opAdd with numpy broadcasting of C against
 * [M, N] (C shape c_shape/c_rank; c == NULL means no C input).
 */
ORC_API int orc_gemm(const float *a, int64_t a_rows, int64_t a_cols, const float *b, int64_t b_rows,
                     int64_t b_cols, const float *c, const int64_t *c_shape, int c_rank, float alpha,
                     float beta, int trans_a, int trans_b, float *y, int nthreads) {
  const int64_t M = trans_a ? a_cols : a_rows, K = trans_a ? a_rows : a_cols;
  const int64_t K2 = trans_b ? b_cols : b_rows, N = trans_b ? b_rows : b_cols;
  if (K != K2) return -1;
  float *at = NULL, *bt = NULL;
  const float *ap = a, *bp = b;
  if (trans_a) {
    at = (float *)malloc(sizeof(float) * (size_t)(M * K + 1));
    for (int64_t i = 0; i < M; i++)
      for (int64_t kk = 0; kk < K; kk++) at[i * K + kk] = a[kk * a_cols + i];
    ap = at;
  }
  if (trans_b) {
    bt = (float *)malloc(sizeof(float) * (size_t)(K * N + 1));
    for (int64_t kk = 0; kk < K; kk++)
      for (int64_t j = 0; j < N; j++) bt[kk * N + j] = b[j * b_cols + kk];
    bp = bt;
  }
  int64_t as[2] = {M, K}, bs[2] = {K, N};
  orc_matmul(ap, as, 2, bp, bs, 2, y, nthreads);
  free(at);
  free(bt);
  if (alpha != 1.0f)
    for (int64_t i = 0; i < M * N; i++) y[i] = y[i] * alpha;
  if (c == NULL) return 0;
  /* C broadcast onto [M, N]: rank <= 2, each dim 1 or equal. */
  int64_t cr = 1, cc = 1;
  if (c_rank == 1) cc = c_shape[0];
  else if (c_rank == 2) {
    cr = c_shape[0];
    cc = c_shape[1];
  } else if (c_rank != 0) return -1;
  if ((cr != 1 && cr != M) || (cc != 1 && cc != N)) return -1;
  for (int64_t i = 0; i < M; i++)
    for (int64_t j = 0; j < N; j++) {
      float cv = c[(cr == 1 ? 0 : i) * cc + (cc == 1 ? 0 : j)];
      if (beta != 1.0f) cv = cv * beta;
      y[i * N + j] = y[i * N + j] + cv;
    }
  return 0;
}

/* ------------------------------------------------------------------------- */
/* opMatMulInteger (onnx_qlinear_ops.dart:32-81)                              */
/* ------------------------------------------------------------------------- */

typedef struct {
  const int32_t *a, *b, *azp, *bzp;
  int64_t *out;
  int64_t batch, a_batch, b_batch, m, k, n, azp_len, bzp_len, j0, j1;
} mmi_job;

static void *mmi_worker(void *p) {
  mmi_job *g = (mmi_job *)p;
  const int64_t m = g->m, k = g->k, n = g->n;
  /* Zero-point rules (:41-44): scalar applies everywhere; a length-M (A) or
   * length-N (B) vector applies per row / column unless M (N) is 1. */
  const int64_t az = (g->azp && g->azp_len == 1) ? g->azp[0] : 0;
  const int32_t *az_row = (g->azp && g->azp_len == m && m != 1) ? g->azp : NULL;
  const int64_t bz = (g->bzp && g->bzp_len == 1) ? g->bzp[0] : 0;
  const int32_t *bz_col = (g->bzp && g->bzp_len == n && n != 1) ? g->bzp : NULL;
  for (int64_t bb = 0; bb < g->batch; bb++) {
    const int64_t a_off = (g->a_batch == 1 ? 0 : bb) * m * k;
    const int64_t b_off = (g->b_batch == 1 ? 0 : bb) * k * n;
    const int64_t o_off = bb * m * n;
    for (int64_t i = 0; i < m; i++) {
      const int64_t azi = az_row ? az_row[i] : az;
      for (int64_t kk = 0; kk < k; kk++) {
        const int64_t av = (int64_t)g->a[a_off + i * k + kk] - azi;
        if (av == 0) continue; /* exact skip (:61-62) */
        const int32_t *brow = g->b + b_off + kk * n;
        int64_t *orow = g->out + o_off + i * n;
        for (int64_t j = g->j0; j < g->j1; j++)
          orow[j] += av * ((int64_t)brow[j] - (bz_col ? (int64_t)bz_col[j] : bz));
      }
    }
  }
  return NULL;
}

static void mmi_set_range(void *p, int64_t j0, int64_t j1) {
  ((mmi_job *)p)->j0 = j0;
  ((mmi_job *)p)->j1 = j1;
}

/* Values of a and b are passed widened to int32 (uint8 / int8 sources).
 * a is [a_batch, m, k], b is [b_batch, k, n]; out is [batch, m, n] int64.
 * Returns -1 on a zero-point shape the reference rejects (:37-40) or a batch
 * mismatch (:47-49). */
ORC_API int orc_matmul_integer(const int32_t *a, int64_t a_batch, int64_t m, int64_t k,
                               const int32_t *b, int64_t b_batch, int64_t n, const int32_t *azp,
                               int64_t azp_len, const int32_t *bzp, int64_t bzp_len, int64_t *out,
                               int nthreads) {
  if ((azp && azp_len != 1 && azp_len != m) || (bzp && bzp_len != 1 && bzp_len != n)) return -1;
  const int64_t batch = a_batch > b_batch ? a_batch : b_batch;
  if ((a_batch != batch && a_batch != 1) || (b_batch != batch && b_batch != 1)) return -1;
  if (batch * m * n > 0) memset(out, 0, sizeof(int64_t) * (size_t)(batch * m * n));
  mmi_job jobs[256];
  for (int t = 0; t < 256; t++) {
    mmi_job g = {a, b, azp, bzp, out, batch, a_batch, b_batch, m, k, n, azp_len, bzp_len, 0, 0};
    jobs[t] = g;
  }
  run_column_split(mmi_worker, jobs, sizeof(mmi_job), n, nthreads, mmi_set_range);
  return 0;
}

/* _roundEven (onnx_qlinear_ops.dart:19-26): ties go to the even integer. */
static int64_t round_even(double v) {
  const double f = floor(v);
  const double frac = v - f;
  if (frac > 0.5) return (int64_t)f + 1;
  if (frac < 0.5) return (int64_t)f;
  const int64_t i = (int64_t)f;
  return (i % 2 == 0) ? i : i + 1;
}

ORC_API int64_t orc_round_even(double v) { return round_even(v); }

/* opDynamicQuantizeLinear (lib/src/onnx_ops.dart:3556-3583): range spans 0;
 * scale and zero point computed in double and stored as float32 where the
 * reference stores through a Float32List; y = clamp(roundEven(f32(x/scale))
 * + zp, 0, 255). Returns the zero point; *scale_out receives the scale. */
ORC_API int64_t orc_dynamic_quantize_linear(const float *x, int64_t n, uint8_t *y, float *scale_out) {
  double mn = 0, mx = 0;
  for (int64_t i = 0; i < n; i++) {
    const double v = x[i];
    if (v < mn) mn = v;
    if (v > mx) mx = v;
  }
  const float scale_f = (float)((mx - mn) / 255.0);
  const double scale = scale_f;
  const float zf32 = scale == 0 ? 0.0f : (float)(-mn / scale);
  double zpf = zf32;
  zpf = zpf < 0.0 ? 0.0 : (zpf > 255.0 ? 255.0 : zpf);
  const int64_t zp = round_even(zpf);
  for (int64_t i = 0; i < n; i++) {
    int64_t q;
    if (scale == 0) {
      q = zp;
    } else {
      const float t = (float)((double)x[i] / scale);
      q = round_even((double)t) + zp;
    }
    y[i] = (uint8_t)(q < 0 ? 0 : (q > 255 ? 255 : q));
  }
  *scale_out = scale_f;
  return zp;
}

/* QLinearMatMul requant multiplier (:95-99): each step rounds to float32. */
ORC_API float orc_qlinear_multiplier(float a_scale, float b_scale, float y_scale) {
  float f = (float)((double)a_scale * (double)b_scale);
  f = (float)((double)f / (double)y_scale);
  return f;
}

/* opQLinearMatMul (:85-108): per-tensor scales; yzp scalar (or absent). */
ORC_API int orc_qlinear_matmul(const int32_t *a, int64_t a_batch, int64_t m, int64_t k,
                               const int32_t *b, int64_t b_batch, int64_t n, const int32_t *azp,
                               int64_t azp_len, const int32_t *bzp, int64_t bzp_len, float a_scale,
                               float b_scale, float y_scale, int32_t y_zp, int32_t lo, int32_t hi,
                               int64_t *out, int nthreads) {
  int rc = orc_matmul_integer(a, a_batch, m, k, b, b_batch, n, azp, azp_len, bzp, bzp_len, out,
                              nthreads);
  if (rc) return rc;
  const double mult = (double)orc_qlinear_multiplier(a_scale, b_scale, y_scale);
  const int64_t batch = a_batch > b_batch ? a_batch : b_batch;
  for (int64_t i = 0; i < batch * m * n; i++) {
    const float f = (float)((double)out[i] * mult); /* f32[0] = ai[i] * mult */
    int64_t q = round_even((double)f) + y_zp;
    out[i] = q < lo ? lo : (q > hi ? hi : q);
  }
  return 0;
}

/* ------------------------------------------------------------------------- */
/* opMatMulNBits (onnx_qlinear_ops.dart:115-228)                              */
/* ------------------------------------------------------------------------- */

typedef struct {
  const float *a;
  const uint8_t *bq;
  const float *scales;
  const uint8_t *zp_u8; /* packed uint4 zero points, or NULL */
  const float *zp_f32;  /* float zero points, or NULL */
  const float *bias;    /* [n] or NULL */
  float *out;
  int64_t m, k, n, block, j0, j1;
} nbits_job;

/* weight(col, kk) (:177-191): nibble q (low nibble for even kk), zero point
 * from the packed nibble (low for even block), the float zp, or 8; the
 * product is formed in double and stored through a Float32List. */
static inline float nbits_weight(const nbits_job *g, int64_t col, int64_t kk) {
  const int64_t nblocks = (g->k + g->block - 1) / g->block;
  const int64_t blob = g->block / 2;
  const int64_t blk = kk / g->block;
  const uint8_t byte = g->bq[(col * nblocks + blk) * blob + (kk % g->block) / 2];
  const int q = (kk & 1) == 0 ? (byte & 15) : (byte >> 4);
  double zp = 8.0;
  if (g->zp_u8) {
    const int64_t zstride = (nblocks + 1) / 2;
    const uint8_t z = g->zp_u8[col * zstride + blk / 2];
    zp = (double)((blk & 1) == 0 ? (z & 15) : (z >> 4));
  } else if (g->zp_f32) {
    zp = (double)g->zp_f32[col * nblocks + blk];
  }
  return (float)(((double)q - zp) * (double)g->scales[col * nblocks + blk]);
}

static void *nbits_worker(void *p) {
  nbits_job *g = (nbits_job *)p;
  const int64_t m = g->m, k = g->k, n = g->n;
  if (m == 1) {
    /* Token decode (:194-205): double accumulation straight from packed bytes. */
    for (int64_t col = g->j0; col < g->j1; col++) {
      double sum = 0.0;
      for (int64_t kk = 0; kk < k; kk++) sum += (double)g->a[kk] * (double)nbits_weight(g, col, kk);
      g->out[col] = (float)(sum + (g->bias ? (double)g->bias[col] : 0.0));
    }
    return NULL;
  }
  /* Prefill (:208-226): dequantize 32-column tiles to float, run matmulKernel
   * on [m x k] . [k x columns], then add bias in double. Threads own whole
   * tiles (j0/j1 are tile-aligned). */
  const int64_t tile_cols = 32;
  float *bt = (float *)malloc(sizeof(float) * (size_t)(k * tile_cols));
  float *tile = (float *)malloc(sizeof(float) * (size_t)(m * tile_cols));
  for (int64_t start = g->j0; start < g->j1; start += tile_cols) {
    const int64_t columns = n - start < tile_cols ? n - start : tile_cols;
    for (int64_t col = 0; col < columns; col++)
      for (int64_t kk = 0; kk < k; kk++) bt[kk * columns + col] = nbits_weight(g, start + col, kk);
    memset(tile, 0, sizeof(float) * (size_t)(m * columns));
    for (int64_t j = 0; j < columns; j++) gemm_column(g->a, k, bt, columns, tile, columns, m, k, columns, j);
    for (int64_t row = 0; row < m; row++)
      for (int64_t col = 0; col < columns; col++)
        g->out[row * n + start + col] =
            (float)((double)tile[row * columns + col] + (g->bias ? (double)g->bias[start + col] : 0.0));
  }
  free(bt);
  free(tile);
  return NULL;
}

static void nbits_set_range(void *p, int64_t j0, int64_t j1) {
  ((nbits_job *)p)->j0 = j0;
  ((nbits_job *)p)->j1 = j1;
}

/* a: [m, k] fp32; bq: [n, ceil(k/block), block/2]; scales: [n*nblocks];
 * zp_u8: [n * ceil(nblocks/2)] or NULL; zp_f32: [n*nblocks] or NULL;
 * bias: [n] or NULL; out: [m, n]. Shape validation is the caller's (the host
 * layer mirrors :126-166). */
ORC_API int orc_matmul_nbits(const float *a, int64_t m, int64_t k, const uint8_t *bq,
                             const float *scales, const uint8_t *zp_u8, const float *zp_f32,
                             const float *bias, int64_t n, int64_t block, float *out, int nthreads) {
  if (k <= 0 || n <= 0 || block < 16 || (block & (block - 1)) != 0) return -1;
  if (m == 0) return 0;
  nbits_job jobs[256];
  for (int t = 0; t < 256; t++) {
    nbits_job g = {a, bq, scales, zp_u8, zp_f32, bias, out, m, k, n, block, 0, 0};
    jobs[t] = g;
  }
  if (m == 1) {
    run_column_split(nbits_worker, jobs, sizeof(nbits_job), n, nthreads, nbits_set_range);
    return 0;
  }
  /* Split whole 32-column tiles across workers. */
  const int64_t tiles = (n + 31) / 32;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > tiles) nthreads = (int)tiles;
  if (nthreads > 256) nthreads = 256;
  pthread_t tid[256];
  int64_t base = tiles / nthreads, rem = tiles % nthreads, t0 = 0;
  for (int t = 0; t < nthreads; t++) {
    int64_t cnt = base + (t < rem ? 1 : 0);
    jobs[t].j0 = t0 * 32;
    jobs[t].j1 = (t0 + cnt) * 32 < n ? (t0 + cnt) * 32 : n;
    t0 += cnt;
  }
  if (nthreads == 1) {
    nbits_worker(&jobs[0]);
    return 0;
  }
  for (int t = 0; t < nthreads; t++) pthread_create(&tid[t], NULL, nbits_worker, &jobs[t]);
  for (int t = 0; t < nthreads; t++) pthread_join(tid[t], NULL);
  return 0;
}

/* Dequantized weight matrix W[n, k] (float32, the values weight() returns);
 * used by tests to build a float reference for the fast tensor-core mode. */
ORC_API void orc_nbits_dequant(const uint8_t *bq, const float *scales, const uint8_t *zp_u8,
                               const float *zp_f32, int64_t k, int64_t n, int64_t block, float *w) {
  nbits_job g = {NULL, bq, scales, zp_u8, zp_f32, NULL, NULL, 0, k, n, block, 0, 0};
  for (int64_t col = 0; col < n; col++)
    for (int64_t kk = 0; kk < k; kk++) w[col * k + kk] = nbits_weight(&g, col, kk);
}

/* ------------------------------------------------------------------------- */
/* Conv (opConv, lib/src/onnx_nn_ops.dart:179-545), without the Winograd      */
/* branch (:241-277), which only the executor selects for initializer 3x3     */
/* stride-1 kernels with >= 1024 output pixels (:779-812).                    */
/* ------------------------------------------------------------------------- */

/*
 * x [n][cin][sp...] with nd = 1..3 spatial dims, w [m][cpg][k...], bias [m]
 * or NULL, pads resolved (begin[nd], end[nd]), out [n][m][osp...].
 *
 * nd == 1 runs as 2-D with a unit height (:200-215). 2-D:
 *   depthwise (cpg == 1 && m / group == 1): each channel is copied into a
 *     zero-padded plane and every tap, padding included, accumulates in
 *     double from the bias (:423-483);
 *   otherwise im2col in chunks of output rows (chunkRows = (8 << 20) floats /
 *     (colRows * ow), at least 1, at most oh; :313-323 with the executor's
 *     workspace rule onnx_graph.dart:1509-1546), matmulKernel(W_g, cols) per
 *     chunk with the chunk as the call's columns (gemm_column above), then the
 *     bias added in float32 (:406-418). A pointwise conv reads x directly
 *     (:293-306); its chunks are addressed here with the channel stride h*w.
 * 3-D walks the kernel taps in order, skipping taps outside the input, and
 * accumulates in double from the bias (:485-530).
 */
static void conv2d_f32(const float *x, int64_t n, int64_t cin, int64_t h, int64_t wd, const float *w,
                       int64_t m, int64_t cpg, int64_t kh, int64_t kw, const float *bias, int64_t sh, int64_t sw,
                       int64_t dh, int64_t dw, int64_t ph, int64_t pw, int64_t pb, int64_t pr, int64_t group,
                       int64_t oh, int64_t ow, float *out) {
  const int64_t mpg = m / group;
  if (cpg == 1 && mpg == 1) {
    const int64_t hp = h + ph + pb, wp = wd + pw + pr;
    double *xpad = (double *)malloc(sizeof(double) * (size_t)(hp * wp));
    for (int64_t b = 0; b < n; b++) {
      for (int64_t om = 0; om < m; om++) {
        for (int64_t i = 0; i < hp * wp; i++) xpad[i] = 0.0;
        const float *xc = x + (b * cin + om) * h * wd;
        for (int64_t yy = 0; yy < h; yy++)
          for (int64_t xx = 0; xx < wd; xx++) xpad[(yy + ph) * wp + pw + xx] = (double)xc[yy * wd + xx];
        const double acc0 = bias ? (double)bias[om] : 0.0;
        const float *wc = w + om * kh * kw;
        float *oc = out + (b * m + om) * oh * ow;
        for (int64_t oy = 0; oy < oh; oy++) {
          for (int64_t ox = 0; ox < ow; ox++) {
            double acc = acc0;
            const int64_t i0 = oy * sh * wp + ox * sw;
            for (int64_t ky = 0; ky < kh; ky++)
              for (int64_t kx = 0; kx < kw; kx++) acc += xpad[i0 + ky * dh * wp + kx * dw] * (double)wc[ky * kw + kx];
            oc[oy * ow + ox] = (float)acc;
          }
        }
      }
    }
    free(xpad);
    return;
  }
  const int64_t col_rows = cpg * kh * kw, col_n = oh * ow;
  int64_t chunk_rows = ((int64_t)8 << 20) / (col_rows * ow);
  if (chunk_rows < 1) chunk_rows = 1;
  if (chunk_rows > oh) chunk_rows = oh;
  float *cols = (float *)malloc(sizeof(float) * (size_t)(col_rows * chunk_rows * ow));
  for (int64_t b = 0; b < n; b++) {
    for (int64_t g = 0; g < group; g++) {
      const float *xg = x + (b * cin + g * cpg) * h * wd;
      const float *wg = w + g * mpg * col_rows;
      float *og = out + (b * m + g * mpg) * col_n;
      for (int64_t row0 = 0; row0 < oh; row0 += chunk_rows) {
        const int64_t rows = row0 + chunk_rows <= oh ? chunk_rows : oh - row0;
        const int64_t chunk_n = rows * ow;
        for (int64_t r = 0; r < col_rows; r++) {
          const int64_t c = r / (kh * kw), ky = (r / kw) % kh, kx = r % kw;
          for (int64_t oyl = 0; oyl < rows; oyl++) {
            const int64_t iy = (row0 + oyl) * sh - ph + ky * dh;
            for (int64_t ox = 0; ox < ow; ox++) {
              const int64_t ix = ox * sw - pw + kx * dw;
              const int inside = iy >= 0 && iy < h && ix >= 0 && ix < wd;
              cols[r * chunk_n + oyl * ow + ox] = inside ? xg[c * h * wd + iy * wd + ix] : 0.0f;
            }
          }
        }
        for (int64_t j = 0; j < chunk_n; j++)
          gemm_column(wg, col_rows, cols, chunk_n, og + row0 * ow, col_n, mpg, col_rows, chunk_n, j);
      }
    }
  }
  free(cols);
  if (bias) {
    for (int64_t b = 0; b < n; b++)
      for (int64_t om = 0; om < m; om++)
        for (int64_t k = 0; k < col_n; k++) {
          float *o = out + (b * m + om) * col_n + k;
          *o = *o + bias[om];
        }
  }
}

ORC_API int orc_conv_f32(const float *x, const int64_t *xshape, int nd, const float *w, const int64_t *kshape,
                         int64_t m, const float *bias, const int64_t *strides, const int64_t *pads,
                         const int64_t *dil, int64_t group, float *out) {
  if (nd < 1 || nd > 3) return -1;
  const int64_t n = xshape[0], cin = xshape[1];
  if (group < 1 || cin % group || m % group) return -2;
  const int64_t cpg = cin / group, mpg = m / group;
  int64_t osp[3];
  for (int a = 0; a < nd; a++) {
    const int64_t window = dil[a] * (kshape[a] - 1) + 1;
    osp[a] = (xshape[2 + a] + pads[a] + pads[nd + a] - window) / strides[a] + 1;
    if (osp[a] < 1) return -3;
  }
  if (nd == 1) {
    conv2d_f32(x, n, cin, 1, xshape[2], w, m, cpg, 1, kshape[0], bias, 1, strides[0], 1, dil[0], 0, pads[0], 0,
               pads[1], group, 1, osp[0], out);
    return 0;
  }
  if (nd == 2) {
    conv2d_f32(x, n, cin, xshape[2], xshape[3], w, m, cpg, kshape[0], kshape[1], bias, strides[0], strides[1],
               dil[0], dil[1], pads[0], pads[1], pads[2], pads[3], group, osp[0], osp[1], out);
    return 0;
  }
  const int64_t in_n = xshape[2] * xshape[3] * xshape[4];
  const int64_t k_n = kshape[0] * kshape[1] * kshape[2];
  const int64_t out_n = osp[0] * osp[1] * osp[2];
  for (int64_t b = 0; b < n; b++) {
    for (int64_t om = 0; om < m; om++) {
      const int64_t g = om / mpg;
      const double acc0 = bias ? (double)bias[om] : 0.0;
      for (int64_t oi = 0; oi < out_n; oi++) {
        const int64_t oc[3] = {oi / (osp[1] * osp[2]), (oi / osp[2]) % osp[1], oi % osp[2]};
        double acc = acc0;
        for (int64_t c = 0; c < cpg; c++) {
          const float *xc = x + (b * cin + g * cpg + c) * in_n;
          const float *wc = w + (om * cpg + c) * k_n;
          for (int64_t ki = 0; ki < k_n; ki++) {
            const int64_t kc[3] = {ki / (kshape[1] * kshape[2]), (ki / kshape[2]) % kshape[1], ki % kshape[2]};
            int64_t off = 0;
            int inside = 1;
            for (int a = 0; a < 3; a++) {
              const int64_t ia = oc[a] * strides[a] - pads[a] + kc[a] * dil[a];
              if (ia < 0 || ia >= xshape[2 + a]) {
                inside = 0;
                break;
              }
              off = off * xshape[2 + a] + ia;
            }
            if (inside) acc += (double)xc[off] * (double)wc[ki];
          }
        }
        out[(b * m + om) * out_n + oi] = (float)acc;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------- */
/* Conv, Winograd F(2x2, 3x3) branch (lib/src/onnx_nn_ops.dart:271-293,       */
/* 584-786)                                                                   */
/* ------------------------------------------------------------------------- */

/*
 * The executor takes this branch for an initializer weight [M, C, 3, 3],
 * group 1, stride 1, dilation 1, symmetric pads all 0 or all 1, with at least
 * 1024 output pixels (convWinogradEligible :779-812, onnx_graph.dart:2450).
 * A standalone call (no isolate pool band), with its arithmetic:
 *   - weights (pretransformWinogradF2x2 :584-628): U[y*4+x][om*C+ic] =
 *     f32(sum over ky, kx of (g[y][ky] * w) * g[x][kx]) in double, ky outer;
 *   - tile rows in bands of max(1, (16 << 20) / (16 (C + M) tw)) rows, tw =
 *     ceil(outW / 2) (:652-660); per band the input rows go into a zeroed
 *     padded buffer of rows*2 + 2 rows by tw*2 + 2 columns, padLeft in;
 *   - input transform (:683-704) in double from the float inputs, each of the
 *     16 planes stored as float: V = Bᵀ d B with the row pass first;
 *   - 16 products: matmulKernel(U[q] [M x C], V[q] [C x band tiles]);
 *   - output transform (:717-746) in double from the float products, the row
 *     pass first (a0 + a1 + a2, a1 - a2 - a3), then the column pass plus the
 *     bias in double, one float rounding per output.
 * Returns 0, or a negative code for shapes the branch does not take.
 */
ORC_API int orc_conv_winograd_f2x2(const float *x, int64_t n, int64_t c, int64_t in_h, int64_t in_w,
                                   const float *w, int64_t m, const float *bias, int64_t pad, float *out) {
  if (pad != 0 && pad != 1) return -1;
  const int64_t out_h = in_h + 2 * pad - 2, out_w = in_w + 2 * pad - 2;
  if (out_h < 1 || out_w < 1 || n < 1 || c < 1 || m < 1) return -2;
  static const double g[4][3] = {{1, 0, 0}, {0.5, 0.5, 0.5}, {0.5, -0.5, 0.5}, {0, 0, 1}};
  float *u = (float *)malloc(sizeof(float) * (size_t)(16 * m * c));
  for (int64_t om = 0; om < m; om++)
    for (int64_t ic = 0; ic < c; ic++) {
      const float *wk = w + (om * c + ic) * 9;
      for (int y = 0; y < 4; y++)
        for (int xx = 0; xx < 4; xx++) {
          double sum = 0;
          for (int ky = 0; ky < 3; ky++)
            for (int kx = 0; kx < 3; kx++) sum += g[y][ky] * (double)wk[ky * 3 + kx] * g[xx][kx];
          u[(size_t)(y * 4 + xx) * (size_t)(m * c) + (size_t)(om * c + ic)] = (float)sum;
        }
    }
  const int64_t tw = (out_w + 1) >> 1, gy1 = (out_h + 1) >> 1;
  int64_t band_rows = ((int64_t)16 << 20) / (16 * (c + m) * tw);
  if (band_rows < 1) band_rows = 1;
  if (band_rows > gy1) band_rows = gy1;
  const int64_t pw = tw * 2 + 2;
  const int64_t max_tiles = band_rows * tw;
  float *padded = (float *)malloc(sizeof(float) * (size_t)(c * (band_rows * 2 + 2) * pw));
  float *v = (float *)malloc(sizeof(float) * (size_t)(16 * c * max_tiles));
  float *prod = (float *)malloc(sizeof(float) * (size_t)(16 * m * max_tiles));
  double tmp[16];
  for (int64_t b = 0; b < n; b++) {
    for (int64_t cy0 = 0; cy0 < gy1; cy0 += band_rows) {
      const int64_t rows = cy0 + band_rows <= gy1 ? band_rows : gy1 - cy0;
      const int64_t tiles = rows * tw, pad_rows = rows * 2 + 2;
      memset(padded, 0, sizeof(float) * (size_t)(c * pad_rows * pw));
      const int64_t row0 = cy0 * 2 - pad;
      for (int64_t ic = 0; ic < c; ic++)
        for (int64_t py = 0; py < pad_rows; py++) {
          const int64_t yy = row0 + py;
          if (yy < 0 || yy >= in_h) continue;
          memcpy(padded + (ic * pad_rows + py) * pw + pad, x + ((b * c + ic) * in_h + yy) * in_w,
                 sizeof(float) * (size_t)in_w);
        }
      for (int64_t ic = 0; ic < c; ic++)
        for (int64_t ty = 0; ty < rows; ty++)
          for (int64_t tx = 0; tx < tw; tx++) {
            for (int r = 0; r < 4; r++) {
              const float *d = padded + (ic * pad_rows + ty * 2 + r) * pw + tx * 2;
              const double d0 = d[0], d1 = d[1], d2 = d[2], d3 = d[3];
              tmp[r * 4 + 0] = d0 - d2;
              tmp[r * 4 + 1] = d1 + d2;
              tmp[r * 4 + 2] = -d1 + d2;
              tmp[r * 4 + 3] = d1 - d3;
            }
            const int64_t tile = ty * tw + tx;
            for (int col = 0; col < 4; col++) {
              const double a0 = tmp[col], a1 = tmp[4 + col], a2 = tmp[8 + col], a3 = tmp[12 + col];
              v[(size_t)col * (size_t)(c * tiles) + (size_t)(ic * tiles + tile)] = (float)(a0 - a2);
              v[(size_t)(4 + col) * (size_t)(c * tiles) + (size_t)(ic * tiles + tile)] = (float)(a1 + a2);
              v[(size_t)(8 + col) * (size_t)(c * tiles) + (size_t)(ic * tiles + tile)] = (float)(-a1 + a2);
              v[(size_t)(12 + col) * (size_t)(c * tiles) + (size_t)(ic * tiles + tile)] = (float)(a1 - a3);
            }
          }
      for (int q = 0; q < 16; q++) {
        const float *uq = u + (size_t)q * (size_t)(m * c);
        const float *vq = v + (size_t)q * (size_t)(c * tiles);
        float *pq = prod + (size_t)q * (size_t)(m * tiles);
        for (int64_t j = 0; j < tiles; j++) gemm_column(uq, c, vq, tiles, pq, tiles, m, c, tiles, j);
      }
      for (int64_t om = 0; om < m; om++) {
        float *ob = out + (b * m + om) * out_h * out_w;
        const double bias0 = bias ? (double)bias[om] : 0.0;
        for (int64_t ty = 0; ty < rows; ty++) {
          const int64_t oy = (cy0 + ty) * 2;
          for (int64_t tx = 0; tx < tw; tx++) {
            const int64_t tile = ty * tw + tx;
            for (int col = 0; col < 4; col++) {
              const double a0 = prod[(size_t)col * (size_t)(m * tiles) + (size_t)(om * tiles + tile)];
              const double a1 = prod[(size_t)(4 + col) * (size_t)(m * tiles) + (size_t)(om * tiles + tile)];
              const double a2 = prod[(size_t)(8 + col) * (size_t)(m * tiles) + (size_t)(om * tiles + tile)];
              const double a3 = prod[(size_t)(12 + col) * (size_t)(m * tiles) + (size_t)(om * tiles + tile)];
              tmp[col] = a0 + a1 + a2;
              tmp[4 + col] = a1 - a2 - a3;
            }
            const int64_t ox = tx * 2;
            if (oy < out_h) {
              if (ox < out_w) ob[oy * out_w + ox] = (float)(tmp[0] + tmp[1] + tmp[2] + bias0);
              if (ox + 1 < out_w) ob[oy * out_w + ox + 1] = (float)(tmp[1] - tmp[2] - tmp[3] + bias0);
            }
            if (oy + 1 < out_h) {
              if (ox < out_w) ob[(oy + 1) * out_w + ox] = (float)(tmp[4] + tmp[5] + tmp[6] + bias0);
              if (ox + 1 < out_w) ob[(oy + 1) * out_w + ox + 1] = (float)(tmp[5] - tmp[6] - tmp[7] + bias0);
            }
          }
        }
      }
    }
  }
  free(u);
  free(padded);
  free(v);
  free(prod);
  return 0;
}

/* ------------------------------------------------------------------------- */
/* ConvInteger / QLinearConv (lib/src/onnx_qlinear_ops.dart:230-382)          */
/* ------------------------------------------------------------------------- */

/* _convIntAcc (:232-291): acc[n,m,oy,ox] = sum over in-range taps of
 * (x - xZp)(w - wZp[m]), exact (int64). 2-D; 1-D callers pass h = kh = 1. */
ORC_API void orc_conv_int_acc(const int32_t *x, int64_t n, int64_t cin, int64_t h, int64_t wd, const int32_t *w,
                              int64_t m, int64_t cpg, int64_t kh, int64_t kw, int32_t xzp, const int32_t *wzp,
                              int64_t sh, int64_t sw, int64_t dh, int64_t dw, int64_t ph, int64_t pw, int64_t group,
                              int64_t oh, int64_t ow, int64_t *out) {
  const int64_t mpg = m / group;
  for (int64_t b = 0; b < n; b++) {
    for (int64_t om = 0; om < m; om++) {
      const int64_t g = om / mpg;
      const int64_t wz = wzp[om];
      for (int64_t oy = 0; oy < oh; oy++) {
        for (int64_t ox = 0; ox < ow; ox++) {
          int64_t acc = 0;
          for (int64_t c = 0; c < cpg; c++) {
            const int32_t *xc = x + (b * cin + g * cpg + c) * h * wd;
            const int32_t *wc = w + (om * cpg + c) * kh * kw;
            for (int64_t ky = 0; ky < kh; ky++) {
              const int64_t iy = oy * sh - ph + ky * dh;
              if (iy < 0 || iy >= h) continue;
              for (int64_t kx = 0; kx < kw; kx++) {
                const int64_t ix = ox * sw - pw + kx * dw;
                if (ix < 0 || ix >= wd) continue;
                acc += (int64_t)(xc[iy * wd + ix] - xzp) * (int64_t)(wc[ky * kw + kx] - wz);
              }
            }
          }
          out[((b * m + om) * oh + oy) * ow + ox] = acc;
        }
      }
    }
  }
}

/* QLinearConv's requantisation (:361-380): mult = xs * ws[om] / ys in double,
 * q = roundEven((acc + bias[om]) * mult) + yz, clamped to [lo, hi]. */
ORC_API void orc_qlinear_conv_requant(const int64_t *acc, int64_t n, int64_t m, int64_t spn, double xs,
                                      const double *ws, int64_t ws_len, double ys, int64_t yz, const int64_t *bias,
                                      int64_t lo, int64_t hi, int64_t *out) {
  for (int64_t b = 0; b < n; b++) {
    for (int64_t om = 0; om < m; om++) {
      const double mult = xs * ws[ws_len == 1 ? 0 : om] / ys;
      const int64_t bv = bias ? bias[om] : 0;
      const int64_t base = (b * m + om) * spn;
      for (int64_t k = 0; k < spn; k++) {
        const int64_t q = round_even((double)(acc[base + k] + bv) * mult) + yz;
        out[base + k] = q < lo ? lo : (q > hi ? hi : q);
      }
    }
  }
}

/* ------------------------------------------------------------------------- */
/* ConvTranspose (opConvTranspose, lib/src/onnx_nn_ops.dart:815-1060)         */
/* ------------------------------------------------------------------------- */

/*
 * x [n][cin][sp...] (nd = 1..3), w [cin][mpg][k...], bias [m] or NULL, pads
 * [begin..., end...], out_shape: the requested spatial output dims or NULL.
 * With n == 1, nd <= 2 and no output_shape the reference takes its GEMM path
 * (:850-963): per group, prod[mpg*kvol][H*W] = matmulKernel(W_g^T, X_g) (the
 * gemm_column rule with m = mpg*kvol, k = cin/group, n = H*W), then an
 * overlap-add of each (mm, kh, kw) plane into the float32 output (loop order
 * mm, kh, kw, ih, iw) and the bias added in float32. Otherwise the generic
 * scatter (:965-1050): for b, c, input position ii, tap ki (ascending), every
 * non-zero input adds v * w in double onto the float32 output element, which
 * is stored back as float32; then the bias. output_shape recomputes the pads
 * (total = full - requested; end = total / 2, begin = total - end).
 */
ORC_API int orc_conv_transpose_f32(const float *x, const int64_t *xshape, int nd, const float *w,
                                   const int64_t *kshape, int64_t mpg, int64_t group, const float *bias,
                                   const int64_t *strides, const int64_t *pads_in, const int64_t *dil,
                                   const int64_t *outpad, const int64_t *out_shape, float *out, int64_t *osp_out) {
  if (nd < 1 || nd > 3) return -1;
  const int64_t n = xshape[0], cin = xshape[1];
  if (group < 1 || cin % group) return -2;
  const int64_t cpg = cin / group, m = mpg * group;
  int64_t p[6], osp[3];
  for (int a = 0; a < 2 * nd; a++) p[a] = pads_in ? pads_in[a] : 0;
  for (int a = 0; a < nd; a++) {
    const int64_t full = (xshape[2 + a] - 1) * strides[a] + dil[a] * (kshape[a] - 1) + 1 + outpad[a];
    if (out_shape) {
      osp[a] = out_shape[a];
      const int64_t total = full - osp[a];
      p[nd + a] = total / 2;
      p[a] = total - p[nd + a];
    } else {
      osp[a] = full - p[a] - p[nd + a];
    }
    if (osp[a] < 1) return -3;
    osp_out[a] = osp[a];
  }
  int64_t in_n = 1, k_n = 1, out_n = 1;
  for (int a = 0; a < nd; a++) {
    in_n *= xshape[2 + a];
    k_n *= kshape[a];
    out_n *= osp[a];
  }
  for (int64_t i = 0; i < n * m * out_n; i++) out[i] = 0.0f;
  if (nd <= 2 && !out_shape && n == 1) {
    const int64_t H = nd == 2 ? xshape[2] : 1, W = xshape[1 + nd], kH = nd == 2 ? kshape[0] : 1,
                  kW = kshape[nd - 1];
    const int64_t sH = nd == 2 ? strides[0] : 1, sW = strides[nd - 1], dH = nd == 2 ? dil[0] : 1,
                  dW = dil[nd - 1];
    const int64_t pT = nd == 2 ? p[0] : 0, pL = nd == 2 ? p[1] : p[0];
    const int64_t oH = nd == 2 ? osp[0] : 1, oW = osp[nd - 1];
    const int64_t hw = H * W, mk = mpg * k_n;
    float *wt = (float *)malloc(sizeof(float) * (size_t)(mk * cpg));
    float *prod = (float *)malloc(sizeof(float) * (size_t)(mk * hw));
    for (int64_t g = 0; g < group; g++) {
      for (int64_t c = 0; c < cpg; c++)
        for (int64_t idx = 0; idx < mk; idx++) wt[idx * cpg + c] = w[(g * cpg + c) * mk + idx];
      for (int64_t j = 0; j < hw; j++) gemm_column(wt, cpg, x + g * cpg * hw, hw, prod, hw, mk, cpg, hw, j);
      for (int64_t mm = 0; mm < mpg; mm++) {
        float *ob = out + (g * mpg + mm) * oH * oW;
        for (int64_t kh = 0; kh < kH; kh++)
          for (int64_t kw = 0; kw < kW; kw++) {
            const float *pb = prod + ((mm * kH + kh) * kW + kw) * hw;
            for (int64_t ih = 0; ih < H; ih++) {
              const int64_t oh = ih * sH + kh * dH - pT;
              if (oh < 0 || oh >= oH) continue;
              for (int64_t iw = 0; iw < W; iw++) {
                const int64_t ow = iw * sW + kw * dW - pL;
                if (ow >= 0 && ow < oW) ob[oh * oW + ow] = ob[oh * oW + ow] + pb[ih * W + iw];
              }
            }
          }
      }
    }
    free(wt);
    free(prod);
  } else {
    int64_t ostr[3] = {1, 1, 1};
    for (int a = nd - 2; a >= 0; a--) ostr[a] = ostr[a + 1] * osp[a + 1];
    for (int64_t b = 0; b < n; b++)
      for (int64_t c = 0; c < cin; c++) {
        const int64_t g = c / cpg;
        for (int64_t ii = 0; ii < in_n; ii++) {
          const float v = x[(b * cin + c) * in_n + ii];
          if (v == 0.0f) continue;
          int64_t ic[3], rem = ii;
          for (int a = nd - 1; a >= 0; a--) {
            ic[a] = rem % xshape[2 + a];
            rem /= xshape[2 + a];
          }
          for (int64_t ki = 0; ki < k_n; ki++) {
            int64_t kc[3], kr = ki, off = 0;
            for (int a = nd - 1; a >= 0; a--) {
              kc[a] = kr % kshape[a];
              kr /= kshape[a];
            }
            int inside = 1;
            for (int a = 0; a < nd; a++) {
              const int64_t oa = ic[a] * strides[a] + kc[a] * dil[a] - p[a];
              if (oa < 0 || oa >= osp[a]) {
                inside = 0;
                break;
              }
              off += oa * ostr[a];
            }
            if (!inside) continue;
            for (int64_t mm = 0; mm < mpg; mm++) {
              float *o = out + (b * m + g * mpg + mm) * out_n + off;
              *o = (float)((double)*o + (double)v * (double)w[(c * mpg + mm) * k_n + ki]);
            }
          }
        }
      }
  }
  if (bias)
    for (int64_t b = 0; b < n; b++)
      for (int64_t om = 0; om < m; om++)
        for (int64_t k = 0; k < out_n; k++) out[(b * m + om) * out_n + k] = out[(b * m + om) * out_n + k] + bias[om];
  return 0;
}
