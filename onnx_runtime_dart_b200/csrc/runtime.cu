// C ABI of libb200mm.so (declared in include/b2m.h): contexts, device
// tensors, weight prepack, operator validation and kernel dispatch.
//
// Validation mirrors the reference's operator functions so the same inputs
// fail with the same class of error: opMatMul / opGemm
// (lib/src/onnx_ops.dart:1710-1766, 2152-2173), opMatMulInteger /
// opQLinearMatMul (lib/src/onnx_qlinear_ops.dart:32-108) and opMatMulNBits
// (:115-228).
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "b2m_internal.cuh"

namespace {

thread_local std::string g_last_error;

template <class F>
b2m_status guarded(F &&f) {
  try {
    f();
    return B2M_OK;
  } catch (const B2mError &e) {
    g_last_error = e.msg;
    return e.code;
  } catch (const std::bad_alloc &) {
    g_last_error = "host allocation failed";
    return B2M_ERR_OUT_OF_MEMORY;
  } catch (...) {
    g_last_error = "unexpected internal error";
    return B2M_ERR_CUDA;
  }
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) B2M_CUDA(cudaSetDevice(dev));
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int64_t elem_size(int32_t dtype) {
  switch (dtype) {
    case B2M_FLOAT: return 4;
    case B2M_UINT8: return 1;
    case B2M_INT8: return 1;
    case B2M_INT32: return 4;
    case B2M_INT64: return 8;
    case B2M_FLOAT16: return 2;
    default: return 0;
  }
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

std::string shape_str(const int64_t *s, int r) {
  std::string o = "[";
  for (int i = 0; i < r; i++) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

void check_ctx(b2m_ctx *ctx) { B2M_REQUIRE(ctx, B2M_ERR_INVALID_ARGUMENT, "null context"); }

void check_cancel(b2m_ctx *ctx) {
  if (ctx->cancel_flag && *ctx->cancel_flag) b2m_throw(B2M_ERR_CANCELLED, "operation cancelled");
}

// Bounded device waits report through the mapped error word; a call that
// has just synchronised the stream reads it with a plain host load.
void raise_device_error(b2m_ctx *ctx) {
  const int32_t e = *reinterpret_cast<volatile int32_t *>(ctx->err_host);
  if (e != B2M_DEVERR_NONE) {
    *reinterpret_cast<volatile int32_t *>(ctx->err_host) = B2M_DEVERR_NONE;
    // An aborted kernel may leave counters mid-count: clear the whole block.
    B2M_CUDA(cudaMemsetAsync(ctx->dev_counter, 0, B2M_DEV_STATE_BYTES, ctx->stream));
    if (e == B2M_DEVERR_INDEX)
      b2m_throw(B2M_ERR_INVALID_ARGUMENT, "an index (a gather id or a rotary position) was outside its table");
    if (e == B2M_DEVERR_CACHE_FULL) b2m_throw(B2M_ERR_INVALID_ARGUMENT, "a KV-cache append went past its capacity");
    b2m_throw(B2M_ERR_TIMEOUT, "a bounded device-side wait timed out (code " + std::to_string(e) + ")");
  }
}

void check_device_error(b2m_ctx *ctx) {
  B2M_CUDA(cudaStreamSynchronize(ctx->stream));
  raise_device_error(ctx);
}

// The device address of a host buffer that kernels can write directly
// (pinned or registered host memory), or nullptr for pageable memory.
void *mapped_host_ptr(void *p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

b2m_tensor *new_tensor(b2m_ctx *ctx, int32_t dtype, const int64_t *shape, int32_t rank) {
  B2M_REQUIRE(rank >= 0 && rank <= B2M_MAX_RANK, B2M_ERR_INVALID_ARGUMENT, "tensor rank out of range");
  B2M_REQUIRE(elem_size(dtype) > 0, B2M_ERR_INVALID_ARGUMENT, "unsupported tensor dtype");
  int64_t numel = 1;
  for (int i = 0; i < rank; i++) {
    B2M_REQUIRE(shape[i] >= 0, B2M_ERR_INVALID_ARGUMENT, "negative dimension");
    numel *= shape[i];
  }
  const int64_t bytes = numel * elem_size(dtype);
  if (ctx->byte_budget > 0 && ctx->live_bytes + bytes > ctx->byte_budget)
    b2m_throw(B2M_ERR_OUT_OF_MEMORY, "tensor byte budget exceeded (" + std::to_string(ctx->live_bytes + bytes) +
                                         " > " + std::to_string(ctx->byte_budget) + ")");
  b2m_tensor *t = new b2m_tensor();
  t->ctx = ctx;
  t->dtype = dtype;
  t->rank = rank;
  for (int i = 0; i < rank; i++) t->shape[i] = shape[i];
  t->numel = numel;
  t->owned = true;
  if (bytes > 0) {
    cudaError_t e = cudaMallocAsync(&t->data, (size_t)bytes, ctx->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      delete t;
      b2m_throw(B2M_ERR_OUT_OF_MEMORY, std::string("device allocation failed: ") + cudaGetErrorString(e));
    }
  }
  ctx->live_bytes += bytes;
  return t;
}

int64_t tensor_bytes(const b2m_tensor *t) { return t->numel * elem_size(t->dtype); }

// Output handling: *y == NULL -> allocate; else check dtype / element count.
b2m_tensor *prepare_output(b2m_ctx *ctx, b2m_tensor **y, int32_t dtype, const std::vector<int64_t> &shape) {
  B2M_REQUIRE(y, B2M_ERR_INVALID_ARGUMENT, "null output pointer");
  if (*y == nullptr) {
    *y = new_tensor(ctx, dtype, shape.data(), (int32_t)shape.size());
    return *y;
  }
  b2m_tensor *t = *y;
  int64_t numel = 1;
  for (int64_t d : shape) numel *= d;
  B2M_REQUIRE(t->dtype == dtype && t->numel == numel, B2M_ERR_INVALID_ARGUMENT,
              "output tensor has the wrong dtype or size for " + shape_str(shape.data(), (int)shape.size()));
  t->rank = (int32_t)shape.size();
  for (size_t i = 0; i < shape.size(); i++) t->shape[i] = shape[i];
  return t;
}

// Bump allocator over the context workspace; reset at the start of each op.
struct Scratch {
  b2m_ctx *ctx;
  size_t used = 0;
  explicit Scratch(b2m_ctx *c, size_t need) : ctx(c) {
    if (need > 0 && need > ctx->scratch_bytes) {
      if (ctx->scratch) B2M_CUDA(cudaFreeAsync(ctx->scratch, ctx->stream));
      ctx->scratch = nullptr;
      ctx->scratch_bytes = 0;
      const size_t sz = std::max(need, (size_t)1 << 20);
      B2M_CUDA(cudaMallocAsync(&ctx->scratch, sz, ctx->stream));
      ctx->scratch_bytes = sz;
    }
  }
  void *take(size_t bytes) {
    const size_t off = (used + 255) & ~(size_t)255;
    B2M_REQUIRE(off + bytes <= ctx->scratch_bytes, B2M_ERR_CUDA, "internal: scratch overflow");
    used = off + bytes;
    return static_cast<char *>(ctx->scratch) + off;
  }
};

struct OpTimer {
  b2m_ctx *ctx;
  explicit OpTimer(b2m_ctx *c) : ctx(c) {
    if (ctx->timing) B2M_CUDA(cudaEventRecord(ctx->ev0, ctx->stream));
  }
  void done() {
    if (ctx->timing) {
      B2M_CUDA(cudaEventRecord(ctx->ev1, ctx->stream));
      ctx->timing_pending = true;
    }
  }
};

void require_float(const b2m_tensor *t, const char *what) {
  B2M_REQUIRE(t, B2M_ERR_INVALID_ARGUMENT, std::string(what) + " is null");
  B2M_REQUIRE(t->dtype == B2M_FLOAT, B2M_ERR_INVALID_ARGUMENT, std::string(what) + " must be float32");
}

// ---------------------------------------------------------------------------
// fp32 MatMul / Gemm
// ---------------------------------------------------------------------------

// Round-to-nearest-even fp32 -> bf16 bits (quiet NaN for NaN).
uint16_t bf16_rn_host(float v) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

float bf16_to_float_host(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// The device split (k_f32_tc.cu): x0 = rn(x) (truncated instead when rounding
// would overflow a finite x), x1 = rn(x - x0), x1 = 0 for non-finite x.
void split_bf16_host(float v, uint16_t &h, uint16_t &l) {
  h = bf16_rn_host(v);
  float hf = bf16_to_float_host(h);
  const bool fin = std::isfinite(v);
  if (std::isinf(hf) && fin) {
    uint32_t u;
    std::memcpy(&u, &v, 4);
    h = (uint16_t)(u >> 16);
    hf = bf16_to_float_host(h);
  }
  l = bf16_rn_host(fin ? v - hf : 0.f);
}

// FAST with a prepacked weight and contiguous A rows runs the bf16-split
// product on the tensor cores; everything else (and EXACT) runs the bit-exact
// kernels.
void run_f32(b2m_ctx *ctx, F32GemmArgs &p, const b2m_weight *bw, int32_t mode) {
  p.dev_err = ctx->dev_err;
  if (mode == B2M_MODE_FAST && f32_tc_eligible(p, bw)) {
    const size_t need = f32_tc_scratch_bytes(p.M, p.K);
    Scratch sc(ctx, need + 256);
    launch_f32_tc(p, *bw, sc.take(need), ctx->stream);
    return;
  }
  launch_f32_exact(p, ctx->stream);
}

void matmul_f32_impl(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b, const b2m_weight *bw, int32_t mode,
                     b2m_tensor **y) {
  require_float(a, "MatMul A");
  B2M_REQUIRE((b == nullptr) != (bw == nullptr), B2M_ERR_INVALID_ARGUMENT, "MatMul: pass exactly one of b, b_packed");
  B2M_REQUIRE(mode == B2M_MODE_EXACT || mode == B2M_MODE_FAST, B2M_ERR_INVALID_ARGUMENT, "MatMul: bad mode");
  int64_t bshape[B2M_MAX_RANK];
  int brank;
  const float *bptr;
  if (b) {
    require_float(b, "MatMul B");
    brank = b->rank;
    for (int i = 0; i < brank; i++) bshape[i] = b->shape[i];
    bptr = static_cast<const float *>(b->data);
  } else {
    B2M_REQUIRE(bw->kind == W_F32, B2M_ERR_INVALID_ARGUMENT, "MatMul: b_packed is not an fp32 weight");
    brank = 2;
    bshape[0] = bw->k;
    bshape[1] = bw->n;
    bptr = bw->f32;
  }
  B2M_REQUIRE(a->rank >= 2 && brank >= 2, B2M_ERR_INVALID_ARGUMENT, "MatMul: operands must have rank >= 2");
  const int64_t m = a->shape[a->rank - 2], k = a->shape[a->rank - 1];
  const int64_t k2 = bshape[brank - 2], n = bshape[brank - 1];
  B2M_REQUIRE(k == k2, B2M_ERR_INVALID_ARGUMENT,
              "MatMul inner dims mismatch: " + std::to_string(k) + " vs " + std::to_string(k2));
  // numpy broadcast of the batch dims (_broadcastShape, onnx_ops.dart:26-44)
  const int ab = a->rank - 2, bb = brank - 2, rank = std::max(ab, bb);
  B2M_REQUIRE(rank <= 6, B2M_ERR_UNSUPPORTED, "MatMul: more than 6 batch dims");
  int64_t ap[6], bp[6], ob[6];
  for (int d = 0; d < rank; d++) {
    ap[d] = d < rank - ab ? 1 : a->shape[d - (rank - ab)];
    bp[d] = d < rank - bb ? 1 : bshape[d - (rank - bb)];
    if (ap[d] == bp[d]) ob[d] = ap[d];
    else if (ap[d] == 1) ob[d] = bp[d];
    else if (bp[d] == 1) ob[d] = ap[d];
    else
      b2m_throw(B2M_ERR_INVALID_ARGUMENT, "Cannot broadcast shapes " + shape_str(a->shape, ab) + " and " +
                                              shape_str(bshape, bb));
  }
  std::vector<int64_t> oshape(ob, ob + rank);
  oshape.push_back(m);
  oshape.push_back(n);
  int64_t batch = 1, bcount = 1;
  for (int d = 0; d < rank; d++) batch *= ob[d];
  for (int d = 0; d < bb; d++) bcount *= bshape[d];
  check_cancel(ctx);
  b2m_tensor *out = prepare_output(ctx, y, B2M_FLOAT, oshape);
  if (batch * m * n == 0) return;
  OpTimer timer(ctx);
  F32GemmArgs p;
  p.A = static_cast<const float *>(a->data);
  p.B = bptr;
  p.Y = static_cast<float *>(out->data);
  p.K = k;
  p.N = n;
  p.sa_k = 1;
  p.sa_m = k;
  p.sb_k = n;
  p.sb_n = 1;
  p.ldy = n;
  p.tile_w = n;
  p.epi = EPI_NONE;
  if (batch > 1 && bcount == 1) {
    // Shared 2-D B: one GEMM over all batches' rows (onnx_ops.dart:1728-1735).
    p.M = batch * m;
    p.m_eff = batch * m;
    p.batch = 1;
  } else {
    p.M = m;
    p.m_eff = m;
    p.batch = batch;
    p.nbd = rank;
    // Row-major strides over each operand's own batch dims.
    int64_t sa = m * k, sb = k * n;
    for (int d = rank - 1; d >= 0; d--) {
      p.bdims[d] = ob[d];
      p.a_bstride[d] = ap[d] == 1 ? 0 : sa;
      p.b_bstride[d] = bp[d] == 1 ? 0 : sb;
      sa *= ap[d];
      sb *= bp[d];
    }
    p.y_bstride = m * n;
  }
  run_f32(ctx, p, bw, mode);
  timer.done();
}

void gemm_f32_impl(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b, const b2m_weight *bw,
                   const b2m_tensor *c, float alpha, float beta, int32_t ta, int32_t tb, int32_t mode,
                   b2m_tensor **y) {
  require_float(a, "Gemm A");
  B2M_REQUIRE((b == nullptr) != (bw == nullptr), B2M_ERR_INVALID_ARGUMENT, "Gemm: pass exactly one of b, b_packed");
  B2M_REQUIRE(mode == B2M_MODE_EXACT || mode == B2M_MODE_FAST, B2M_ERR_INVALID_ARGUMENT, "Gemm: bad mode");
  B2M_REQUIRE(a->rank == 2, B2M_ERR_INVALID_ARGUMENT, "Gemm: A must be 2-D");
  int64_t br, bc;
  const float *bptr;
  if (b) {
    require_float(b, "Gemm B");
    B2M_REQUIRE(b->rank == 2, B2M_ERR_INVALID_ARGUMENT, "Gemm: B must be 2-D");
    br = b->shape[0];
    bc = b->shape[1];
    bptr = static_cast<const float *>(b->data);
  } else {
    B2M_REQUIRE(bw->kind == W_F32, B2M_ERR_INVALID_ARGUMENT, "Gemm: b_packed is not an fp32 weight");
    B2M_REQUIRE(!tb, B2M_ERR_INVALID_ARGUMENT, "Gemm: b_packed already holds B' (trans_b must be 0)");
    br = bw->k;
    bc = bw->n;
    bptr = bw->f32;
  }
  const int64_t M = ta ? a->shape[1] : a->shape[0], K = ta ? a->shape[0] : a->shape[1];
  const int64_t K2 = tb ? bc : br, N = tb ? br : bc;
  B2M_REQUIRE(K == K2, B2M_ERR_INVALID_ARGUMENT,
              "MatMul inner dims mismatch: " + std::to_string(K) + " vs " + std::to_string(K2));
  int64_t crs = 0, ccs = 0;
  if (c) {
    require_float(c, "Gemm C");
    int64_t cr = 1, cc = 1;
    if (c->rank == 1) cc = c->shape[0];
    else if (c->rank == 2) {
      cr = c->shape[0];
      cc = c->shape[1];
    } else
      B2M_REQUIRE(c->rank == 0, B2M_ERR_INVALID_ARGUMENT, "Gemm: C must have rank <= 2");
    B2M_REQUIRE((cr == 1 || cr == M) && (cc == 1 || cc == N), B2M_ERR_INVALID_ARGUMENT,
                "Cannot broadcast shapes [" + std::to_string(M) + ", " + std::to_string(N) + "] and " +
                    shape_str(c->shape, c->rank));
    crs = cr == 1 ? 0 : cc;
    ccs = cc == 1 ? 0 : 1;
  }
  check_cancel(ctx);
  b2m_tensor *out = prepare_output(ctx, y, B2M_FLOAT, {M, N});
  if (M * N == 0) return;
  OpTimer timer(ctx);
  F32GemmArgs p;
  p.A = static_cast<const float *>(a->data);
  p.B = bptr;
  p.Y = static_cast<float *>(out->data);
  p.M = M;
  p.N = N;
  p.K = K;
  // A' / B' by strides: the reference's transposes are exact copies.
  const int64_t acols = a->shape[1];
  p.sa_m = ta ? 1 : acols;
  p.sa_k = ta ? acols : 1;
  p.sb_k = tb ? bc : bc;
  p.sb_n = 1;
  if (tb) {
    p.sb_k = 1;
    p.sb_n = bc;
  } else {
    p.sb_k = bc;
    p.sb_n = 1;
  }
  p.ldy = N;
  p.m_eff = M;
  p.tile_w = N;
  p.batch = 1;
  p.epi = EPI_GEMM;
  p.has_alpha = alpha != 1.0f;
  p.alpha = alpha;
  if (c) {
    p.C = static_cast<const float *>(c->data);
    p.c_rs = crs;
    p.c_cs = ccs;
    p.has_beta = beta != 1.0f;
    p.beta = beta;
  }
  run_f32(ctx, p, bw, mode);
  timer.done();
}

// ---------------------------------------------------------------------------
// MatMulInteger / QLinearMatMul
// ---------------------------------------------------------------------------

bool is_i8(int32_t dt) { return dt == B2M_UINT8 || dt == B2M_INT8; }

void integer_impl(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b, const b2m_weight *bw,
                  const b2m_tensor *azp, const b2m_tensor *bzp, bool requant, double mult, int32_t yzp, int32_t lo,
                  int32_t hi, b2m_tensor **y) {
  const char *op = requant ? "QLinearMatMul" : "MatMulInteger";
  B2M_REQUIRE(a && is_i8(a->dtype), B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": A must be uint8 or int8");
  B2M_REQUIRE((b == nullptr) != (bw == nullptr), B2M_ERR_INVALID_ARGUMENT,
              std::string(op) + ": pass exactly one of b, b_packed");
  B2M_REQUIRE(a->rank >= 2, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": A must have rank >= 2");
  const int64_t m = a->shape[a->rank - 2], k = a->shape[a->rank - 1];
  int64_t n, kb, b_batch;
  int32_t bdt;
  if (b) {
    B2M_REQUIRE(is_i8(b->dtype), B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": B must be uint8 or int8");
    B2M_REQUIRE(b->rank >= 2, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": B must have rank >= 2");
    n = b->shape[b->rank - 1];
    kb = b->shape[b->rank - 2];
    b_batch = (kb * n) ? b->numel / (kb * n) : 1;
    bdt = b->dtype;
  } else {
    B2M_REQUIRE(bw->kind == W_I8, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": b_packed is not an int8 weight");
    n = bw->n;
    kb = bw->k;
    b_batch = 1;
    bdt = bw->i8.dtype;
  }
  B2M_REQUIRE(kb == k, B2M_ERR_INVALID_ARGUMENT, std::string(op) + " inner dim mismatch");
  // Zero points: scalar, per-row [M] for A, per-column [N] for B (:37-40).
  if ((azp && azp->numel != 1 && azp->numel != m) || (bzp && bzp->numel != 1 && bzp->numel != n))
    b2m_throw(B2M_ERR_UNSUPPORTED,
              "MatMulInteger: zero points must be scalar, per-row [M] for A or per-column [N] for B");
  if (azp) B2M_REQUIRE(is_i8(azp->dtype), B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": a_zero_point dtype");
  if (bzp) B2M_REQUIRE(is_i8(bzp->dtype), B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": b_zero_point dtype");
  const int64_t a_batch = (m * k) ? a->numel / (m * k) : 1;
  const int64_t batch = std::max(a_batch, b_batch);
  B2M_REQUIRE((a_batch == batch || a_batch == 1) && (b_batch == batch || b_batch == 1), B2M_ERR_INVALID_ARGUMENT,
              std::string(op) + " batch mismatch");
  B2M_REQUIRE(k <= 33025, B2M_ERR_UNSUPPORTED, std::string(op) + ": K > 33025 may leave the int32 range");
  std::vector<int64_t> oshape;
  if (a_batch >= b_batch) oshape.assign(a->shape, a->shape + a->rank - 2);
  else oshape.assign(b->shape, b->shape + b->rank - 2);
  oshape.push_back(m);
  oshape.push_back(n);
  int32_t odt = B2M_INT32;
  if (requant) {
    B2M_REQUIRE((lo == 0 && hi == 255) || (lo == -128 && hi == 127), B2M_ERR_INVALID_ARGUMENT,
                "QLinearMatMul: lo/hi must be [0,255] or [-128,127]");
    odt = lo == 0 ? B2M_UINT8 : B2M_INT8;
  }
  check_cancel(ctx);
  b2m_tensor *out = prepare_output(ctx, y, odt, oshape);
  if (batch * m * n == 0) return;
  OpTimer timer(ctx);
  I8GemmArgs p;
  p.A = a->data;
  p.a_signed = a->dtype == B2M_INT8;
  p.a_bstride = a_batch == 1 ? 0 : m * k;
  p.b_signed = bdt == B2M_INT8;
  p.M = m;
  p.N = n;
  p.K = k;
  p.batch = batch;
  if (bw) {
    p.Bt = bw->i8.bt;
    p.kpad = bw->i8.kpad;
    p.colsum = bw->i8.colsum;
    p.b_bstride = 0;
    p.colsum_bstride = 0;
  } else {
    const int64_t kpad = round_up(std::max<int64_t>(k, 1), 64), npad = round_up(std::max<int64_t>(n, 1), 128);
    Scratch sc(ctx, (size_t)(b_batch * npad * kpad + b_batch * n * 4 + 1024));
    int8_t *bt = static_cast<int8_t *>(sc.take((size_t)(b_batch * npad * kpad)));
    int32_t *cs = static_cast<int32_t *>(sc.take((size_t)(b_batch * n * 4)));
    launch_i8_pack(b->data, p.b_signed, b_batch, k, n, bt, kpad, npad, cs, ctx->stream);
    p.Bt = bt;
    p.kpad = kpad;
    p.colsum = cs;
    p.b_bstride = b_batch == 1 ? 0 : npad * kpad;
    p.colsum_bstride = b_batch == 1 ? 0 : n;
  }
  if (azp) {
    p.azp = azp->data;
    p.azp_len = azp->numel;
    p.azp_signed = azp->dtype == B2M_INT8;
  }
  if (bzp) {
    p.bzp = bzp->data;
    p.bzp_len = bzp->numel;
    p.bzp_signed = bzp->dtype == B2M_INT8;
  }
  if (requant) {
    p.requant = 1;
    p.mult = mult;
    p.y_zp = yzp;
    p.lo = lo;
    p.hi = hi;
    p.Yq = out->data;
  } else {
    p.Y32 = static_cast<int32_t *>(out->data);
  }
  p.dev_err = ctx->dev_err;
  bool done = false;
  if (bw && batch == 1) {
    Scratch rs(ctx, (size_t)m * 4 + 256);
    p.rowsum = static_cast<int32_t *>(rs.take((size_t)m * 4));
    // The declared next call's packed int8 weight goes to L2 (its ts8 layout,
    // which both int8 kernels read).
    const auto it = ctx->next_of.find(bw);
    if (it != ctx->next_of.end() && it->second && it->second->kind == W_I8 && it->second->i8.ts8) {
      p.pf.seg[0] = it->second->i8.ts8;
      p.pf.bytes[0] = it->second->i8.npad * it->second->i8.k128;
    }
    done = launch_i8_tc(p, bw->i8, ctx->stream);
  }
  if (!done) launch_i8_gemm(p, ctx->stream);
  timer.done();
}

// ---------------------------------------------------------------------------
// MatMulNBits
// ---------------------------------------------------------------------------

// FAST route for m rows: the decode GEMV serves m <= 32, except that from 17
// rows on (four m16 tiles per CTA) the tensor-core kernel is faster once the
// GEMV grid (16 columns per CTA) passes 256 CTAs. Measured per op, K = 1024,
// GEMV against tensor cores: N = 4096: m = 24 7.47 / 7.48 us, m = 32 8.16 /
// 7.57 us; N = 6144: m = 24 11.06 / 8.37 us, m = 32 12.00 / 8.19 us; N = 1024
// stays with the GEMV (3.54 / 6.79 us at m = 32). The comparison holds for
// weights with the prefill scale records (tsq); others keep the GEMV.
static bool nbits_use_smallm(const NbitsWeight &w, int64_t m, int64_t K, int64_t N) {
  if (!nbits_smallm_supported(w, m)) return false;
  return !(m > 16 && w.npad >= 4096 && w.tsq && nbits_tc_supported(w, m, K, N));
}

// PRECISE mode: the decode GEMV wherever it serves the row count (exact
// integer weights, fp32 scales, f16 hi + lo activations), otherwise the FAST
// fp32 GEMM (three bf16 products) over the exactly dequantized weight split
// into bf16 planes.
static bool nbits_precise_gemv(const NbitsWeight &w, int64_t m) { return nbits_smallm_supported(w, m); }

static F32GemmArgs nbits_precise_args(const float *A, int64_t m, int64_t K, int64_t N, const float *bias, float *Y) {
  F32GemmArgs p;
  p.A = A;
  p.Y = Y;
  p.M = m;
  p.N = N;
  p.K = K;
  p.sa_m = K;
  p.sa_k = 1;
  p.ldy = N;
  p.batch = 1;
  p.epi = EPI_GEMM;  // y = acc + bias[col]
  p.C = bias;
  p.c_rs = 0;
  p.c_cs = 1;
  return p;
}

// The L2 prefetch plan of an m-row call of `w` in `mode`: the segments the
// same route would read for w's declared successor (decode records for the
// GEMV, the TMEM-operand layout for the tensor-core prefill); none without a
// successor or for other routes.
static void nbits_prefetch_plan(const b2m_ctx *ctx, const b2m_weight *w, int64_t m, int32_t mode, NbitsArgs &p) {
  const auto it = ctx->next_of.find(w);
  if (it == ctx->next_of.end() || !it->second || it->second->kind != W_NBITS) return;
  const b2m_weight *nx = it->second;
  const NbitsWeight &n = nx->nb;
  const bool gemv = mode == B2M_MODE_PRECISE ? nbits_smallm_supported(n, m)
                                             : mode == B2M_MODE_FAST && nbits_use_smallm(n, m, nx->k, nx->n);
  if (gemv && n.drec) {
    p.pf.seg[0] = n.drec;
    p.pf.bytes[0] = (n.npad / 16) * (n.kp / 64) * DREC_BYTES;
  } else if (!gemv && mode == B2M_MODE_FAST && n.tsq && nbits_tc_supported(n, m, nx->k, nx->n)) {
    p.pf.seg[0] = n.tsq;
    p.pf.bytes[0] = (n.npad / 128) * (n.kp / 64) * 4096;
    p.pf.seg[1] = n.tss;
    p.pf.bytes[1] = (n.npad / 128) * (n.kp / 64) * 128 * 8;
  }
}

// Device scratch bytes nbits_run needs for an m-row call.
size_t nbits_scratch_bytes(const b2m_weight *w, int64_t m, int32_t mode) {
  if (m == 0) return 0;
  if (mode == B2M_MODE_PRECISE) {
    if (nbits_precise_gemv(w->nb, m)) return 0;
    return f32_tc_scratch_bytes(m, w->k) + 256;
  }
  if (mode != B2M_MODE_FAST || nbits_use_smallm(w->nb, m, w->k, w->n)) return 0;
  if (!nbits_tc_supported(w->nb, m, w->k, w->n)) return 0;
  return (size_t)(m * nbits_tc_k8(w->k) * 2) + 256;
}

void nbits_run(b2m_ctx *ctx, Scratch &sc, const float *A, int64_t m, const b2m_weight *w, const float *bias,
               int32_t mode, float *Y) {
  B2M_REQUIRE(w && w->kind == W_NBITS, B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: weight is not a MatMulNBits weight");
  B2M_REQUIRE(mode == B2M_MODE_EXACT || mode == B2M_MODE_FAST || mode == B2M_MODE_PRECISE,
              B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: bad mode");
  if (m == 0) return;
  const int64_t K = w->k, N = w->n;
  if (mode == B2M_MODE_PRECISE) {
    if (nbits_precise_gemv(w->nb, m)) {
      NbitsArgs p;
      p.A = A;
      p.w = &w->nb;
      p.bias = bias;
      p.Y = Y;
      p.M = m;
      p.K = K;
      p.N = N;
      p.dev_err = ctx->dev_err;
      nbits_prefetch_plan(ctx, w, m, mode, p);
      launch_nbits_smallm(p, ctx->stream, ctx->pdl);
      return;
    }
    F32GemmArgs p = nbits_precise_args(A, m, K, N, bias, Y);
    p.dev_err = ctx->dev_err;
    B2M_REQUIRE(f32_tc_shape_ok(p), B2M_ERR_UNSUPPORTED, "MatMulNBits: shape not supported in PRECISE mode");
    NbitsWeight &nb = const_cast<b2m_weight *>(w)->nb;
    if (!nb.px_hi) {
      const int64_t kp = f32_tc_kp(K);
      const size_t bytes = (size_t)(N * kp * 2);
      uint16_t *hi = nullptr, *lo = nullptr;
      B2M_CUDA(cudaMalloc(&hi, bytes));
      const cudaError_t e = cudaMalloc(&lo, bytes);
      if (e != cudaSuccess) {
        cudaFree(hi);
        B2M_CUDA(e);
      }
      launch_nbits_split_planes(nb, K, N, kp, hi, lo, ctx->stream);
      nb.px_hi = hi;
      nb.px_lo = lo;
    }
    launch_f32_tc_b(p, nb.px_hi, nb.px_lo, N, sc.take(f32_tc_scratch_bytes(m, K)), ctx->stream);
    return;
  }
  if (mode == B2M_MODE_FAST) {
    NbitsArgs p;
    p.A = A;
    p.w = &w->nb;
    p.bias = bias;
    p.Y = Y;
    p.M = m;
    p.K = K;
    p.N = N;
    p.dev_err = ctx->dev_err;
    nbits_prefetch_plan(ctx, w, m, mode, p);
    if (nbits_use_smallm(w->nb, m, K, N)) {
      launch_nbits_smallm(p, ctx->stream, ctx->pdl);
    } else if (nbits_tc_supported(w->nb, m, K, N)) {
      __half *a16 = static_cast<__half *>(sc.take((size_t)(m * nbits_tc_k8(K) * 2)));

      launch_nbits_tc(p, a16, ctx->stream);
    } else {
      launch_nbits_simt(p, ctx->stream);
    }
    return;
  }
  // EXACT: dequantize once (exactly as weight() does), then the exact GEMM.
  NbitsWeight &nb = const_cast<b2m_weight *>(w)->nb;
  if (!nb.wdeq) {
    B2M_CUDA(cudaMalloc(&nb.wdeq, (size_t)(N * K * 4)));
    launch_nbits_dequant_f32(nb, K, N, nb.wdeq, ctx->stream);
  }
  F32GemmArgs p;
  p.A = A;
  p.B = nb.wdeq;
  p.Y = Y;
  p.M = m;
  p.N = N;
  p.K = K;
  p.sa_m = K;
  p.sa_k = 1;
  p.sb_k = 1;  // B(k, j) = W[j][k]
  p.sb_n = K;
  p.ldy = N;
  p.batch = 1;
  p.bias = bias;
  if (m == 1) {
    p.all_double = 1;  // decode path: double accumulation (:194-205)
    p.m_eff = 1;
    p.tile_w = 32;
    p.epi = EPI_NBITS_M1;
  } else {
    p.m_eff = m;       // 32-column tiles through matmulKernel (:208-226)
    p.tile_w = 32;
    p.epi = EPI_NBITS;
  }
  launch_f32_exact(p, ctx->stream);
}

}  // namespace

[[noreturn]] void b2m_throw(b2m_status code, const std::string &msg) { throw B2mError{code, msg}; }

void b2m_set_last_error(const std::string &msg) { g_last_error = msg; }

// ===========================================================================
// Exported C ABI
// ===========================================================================
extern "C" {

B2M_API int32_t b2m_abi_version(void) { return B2M_ABI_VERSION; }

B2M_API const char *b2m_last_error(void) { return g_last_error.c_str(); }

B2M_API b2m_status b2m_device_count(int32_t *count) {
  return guarded([&] {
    B2M_REQUIRE(count, B2M_ERR_INVALID_ARGUMENT, "null count");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    *count = n;
  });
}

B2M_API b2m_status b2m_init(int32_t device, b2m_ctx **out_ctx) {
  return guarded([&] {
    B2M_REQUIRE(out_ctx, B2M_ERR_INVALID_ARGUMENT, "null out_ctx");
    *out_ctx = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
      (void)cudaGetLastError();
      b2m_throw(B2M_ERR_NO_DEVICE, "no CUDA device available");
    }
    B2M_REQUIRE(device >= 0 && device < n, B2M_ERR_NO_DEVICE, "device ordinal out of range");
    cudaDeviceProp prop;
    B2M_CUDA(cudaGetDeviceProperties(&prop, device));
    B2M_REQUIRE(prop.major == 10 && prop.minor == 0, B2M_ERR_NO_DEVICE,
                std::string("libb200mm is built for sm_100a (B200); device is ") + prop.name);
    DeviceGuard dg(device);
    b2m_ctx *ctx = new b2m_ctx();
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    B2M_CUDA(cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking));
    ctx->stream = ctx->own_stream;
    B2M_CUDA(cudaDeviceGetDefaultMemPool(&ctx->pool, device));
    uint64_t thr = UINT64_MAX;
    B2M_CUDA(cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &thr));
    B2M_CUDA(cudaEventCreate(&ctx->ev0));
    B2M_CUDA(cudaEventCreate(&ctx->ev1));
    // Counters that kernels reset themselves after use (the
    // DynamicQuantizeLinear block counter), and the error word in mapped
    // pinned host memory.
    B2M_CUDA(cudaMalloc(&ctx->dev_counter, B2M_DEV_STATE_BYTES));
    B2M_CUDA(cudaMemset(ctx->dev_counter, 0, B2M_DEV_STATE_BYTES));
    B2M_CUDA(cudaHostAlloc(reinterpret_cast<void **>(&ctx->err_host), sizeof(int32_t), cudaHostAllocMapped));
    *ctx->err_host = B2M_DEVERR_NONE;
    B2M_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void **>(&ctx->dev_err), ctx->err_host, 0));

    const char *no_pdl = std::getenv("B2M_DISABLE_PDL");
    ctx->pdl = !(no_pdl && no_pdl[0] == '1');
    *out_ctx = ctx;
  });
}

B2M_API b2m_status b2m_shutdown(b2m_ctx *ctx) {
  return guarded([&] {
    if (!ctx) return;
    DeviceGuard dg(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaStreamSynchronize(ctx->own_stream);
    if (ctx->scratch) cudaFreeAsync(ctx->scratch, ctx->own_stream);
    cudaStreamSynchronize(ctx->own_stream);
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    cudaFree(ctx->dev_counter);
    cudaFree(ctx->attn_counters);
    cudaEventDestroy(ctx->ev0);
    cudaEventDestroy(ctx->ev1);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
  });
}

B2M_API b2m_status b2m_set_stream(b2m_ctx *ctx, void *stream) {
  return guarded([&] {
    check_ctx(ctx);
    ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  });
}

B2M_API b2m_status b2m_set_attention_mode(b2m_ctx *ctx, int32_t mode) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(mode == B2M_MODE_EXACT || mode == B2M_MODE_FAST, B2M_ERR_INVALID_ARGUMENT,
                "attention mode must be EXACT or FAST");
    ctx->attn_exact = mode == B2M_MODE_EXACT;
  });
}

B2M_API b2m_status b2m_synchronize(b2m_ctx *ctx) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    B2M_CUDA(cudaStreamSynchronize(ctx->stream));
    check_device_error(ctx);
  });
}

B2M_API b2m_status b2m_set_cancel_flag(b2m_ctx *ctx, const volatile int32_t *flag) {
  return guarded([&] {
    check_ctx(ctx);
    ctx->cancel_flag = flag;
  });
}

B2M_API b2m_status b2m_set_byte_budget(b2m_ctx *ctx, int64_t bytes) {
  return guarded([&] {
    check_ctx(ctx);
    ctx->byte_budget = bytes;
  });
}

B2M_API b2m_status b2m_enable_timing(b2m_ctx *ctx, int32_t on) {
  return guarded([&] {
    check_ctx(ctx);
    ctx->timing = on != 0;
  });
}

B2M_API b2m_status b2m_last_kernel_ms(b2m_ctx *ctx, float *ms) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(ms, B2M_ERR_INVALID_ARGUMENT, "null ms");
    DeviceGuard dg(ctx->device);
    if (ctx->timing_pending) {
      B2M_CUDA(cudaEventSynchronize(ctx->ev1));
      B2M_CUDA(cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1));
      ctx->timing_pending = false;
    }
    *ms = ctx->last_ms;
  });
}

// ---- tensors --------------------------------------------------------------

B2M_API b2m_status b2m_tensor_alloc(b2m_ctx *ctx, int32_t dtype, const int64_t *shape, int32_t rank,
                                    b2m_tensor **out) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(out && (shape || rank == 0), B2M_ERR_INVALID_ARGUMENT, "null argument");
    DeviceGuard dg(ctx->device);
    *out = new_tensor(ctx, dtype, shape, rank);
  });
}

B2M_API b2m_status b2m_tensor_wrap(b2m_ctx *ctx, void *device_ptr, int32_t dtype, const int64_t *shape,
                                   int32_t rank, b2m_tensor **out) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(out && (shape || rank == 0), B2M_ERR_INVALID_ARGUMENT, "null argument");
    B2M_REQUIRE(rank >= 0 && rank <= B2M_MAX_RANK, B2M_ERR_INVALID_ARGUMENT, "tensor rank out of range");
    B2M_REQUIRE(elem_size(dtype) > 0, B2M_ERR_INVALID_ARGUMENT, "unsupported tensor dtype");
    b2m_tensor *t = new b2m_tensor();
    t->ctx = ctx;
    t->data = device_ptr;
    t->dtype = dtype;
    t->rank = rank;
    int64_t numel = 1;
    for (int i = 0; i < rank; i++) {
      t->shape[i] = shape[i];
      numel *= shape[i];
    }
    t->numel = numel;
    t->owned = false;
    if (numel > 0 && !device_ptr) {
      delete t;
      b2m_throw(B2M_ERR_INVALID_ARGUMENT, "null device pointer for a non-empty tensor");
    }
    *out = t;
  });
}

B2M_API b2m_status b2m_tensor_upload(b2m_ctx *ctx, b2m_tensor *t, const void *host, int64_t bytes) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(t && (host || bytes == 0), B2M_ERR_INVALID_ARGUMENT, "null argument");
    B2M_REQUIRE(bytes == tensor_bytes(t), B2M_ERR_INVALID_ARGUMENT, "upload size does not match the tensor");
    DeviceGuard dg(ctx->device);
    if (bytes) B2M_CUDA(cudaMemcpyAsync(t->data, host, (size_t)bytes, cudaMemcpyHostToDevice, ctx->stream));
    B2M_CUDA(cudaStreamSynchronize(ctx->stream));
  });
}

B2M_API b2m_status b2m_tensor_download(b2m_ctx *ctx, const b2m_tensor *t, void *host, int64_t bytes) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(t && (host || bytes == 0), B2M_ERR_INVALID_ARGUMENT, "null argument");
    B2M_REQUIRE(bytes == tensor_bytes(t), B2M_ERR_INVALID_ARGUMENT, "download size does not match the tensor");
    DeviceGuard dg(ctx->device);
    if (bytes) B2M_CUDA(cudaMemcpyAsync(host, t->data, (size_t)bytes, cudaMemcpyDeviceToHost, ctx->stream));
    B2M_CUDA(cudaStreamSynchronize(ctx->stream));
    check_device_error(ctx);
  });
}

B2M_API b2m_status b2m_host_alloc(b2m_ctx *ctx, int64_t bytes, void **out) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(out && bytes >= 0, B2M_ERR_INVALID_ARGUMENT, "host alloc: bad arguments");
    *out = nullptr;
    DeviceGuard dg(ctx->device);
    const cudaError_t e = cudaHostAlloc(out, (size_t)std::max<int64_t>(bytes, 1), cudaHostAllocDefault);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      *out = nullptr;
      b2m_throw(B2M_ERR_OUT_OF_MEMORY, "host alloc: cudaHostAlloc of " + std::to_string((long long)bytes) +
                                           " bytes failed");
    }
  });
}

B2M_API b2m_status b2m_host_free(b2m_ctx *ctx, void *p) {
  return guarded([&] {
    check_ctx(ctx);
    if (!p) return;
    DeviceGuard dg(ctx->device);
    B2M_CUDA(cudaFreeHost(p));
  });
}

B2M_API b2m_status b2m_tensor_free(b2m_tensor *t) {
  return guarded([&] {
    if (!t) return;
    if (t->owned && t->data) {
      DeviceGuard dg(t->ctx->device);
      B2M_CUDA(cudaFreeAsync(t->data, t->ctx->stream));
      t->ctx->live_bytes -= tensor_bytes(t);
    }
    delete t;
  });
}

B2M_API b2m_status b2m_tensor_info(const b2m_tensor *t, int32_t *dtype, int32_t *rank, int64_t *shape,
                                   void **device_ptr) {
  return guarded([&] {
    B2M_REQUIRE(t, B2M_ERR_INVALID_ARGUMENT, "null tensor");
    if (dtype) *dtype = t->dtype;
    if (rank) *rank = t->rank;
    if (shape)
      for (int i = 0; i < B2M_MAX_RANK; i++) shape[i] = i < t->rank ? t->shape[i] : 0;
    if (device_ptr) *device_ptr = t->data;
  });
}

// ---- weights --------------------------------------------------------------

B2M_API b2m_status b2m_weight_prepack_f32(b2m_ctx *ctx, const float *host_b, int64_t rows, int64_t cols,
                                          int32_t trans, b2m_weight **out) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(out && host_b && rows > 0 && cols > 0, B2M_ERR_INVALID_ARGUMENT, "Gemm prepack: bad arguments");
    DeviceGuard dg(ctx->device);
    const int64_t K = trans ? cols : rows, N = trans ? rows : cols;
    std::vector<float> packed;
    const float *src = host_b;
    if (trans) {  // opTranspose(B, [1, 0]) once (onnx_graph.dart:2159-2161)
      packed.resize((size_t)(K * N));
      for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++) packed[(size_t)(c * N + r)] = host_b[r * cols + c];
      src = packed.data();
    }
    b2m_weight *w = new b2m_weight();
    w->ctx = ctx;
    w->kind = W_F32;
    w->k = K;
    w->n = N;
    cudaError_t e = cudaMalloc(&w->f32, (size_t)(K * N * 4));
    w->seg_bytes[SEG_F32] = (size_t)(K * N * 4);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      delete w;
      b2m_throw(B2M_ERR_OUT_OF_MEMORY, "weight allocation failed");
    }
    B2M_CUDA(cudaMemcpy(w->f32, src, (size_t)(K * N * 4), cudaMemcpyHostToDevice));
    // bf16 split planes for FAST mode (k_f32_tc.cu): x0 = rn(x), x1 = rn(x - x0),
    // K-major, K padded to 64.
    {
      const int64_t kp = f32_tc_kp(K);
      std::vector<uint16_t> hi((size_t)(N * kp), 0), lo((size_t)(N * kp), 0);
      for (int64_t kk = 0; kk < K; kk++)
        for (int64_t j = 0; j < N; j++) {
          uint16_t h, l;
          split_bf16_host(src[kk * N + j], h, l);
          hi[(size_t)(j * kp + kk)] = h;
          lo[(size_t)(j * kp + kk)] = l;
        }
      cudaError_t e1 = cudaMalloc(&w->bx_hi, hi.size() * 2);
      cudaError_t e2 = e1 == cudaSuccess ? cudaMalloc(&w->bx_lo, lo.size() * 2) : e1;
      if (e1 != cudaSuccess || e2 != cudaSuccess) {
        (void)cudaGetLastError();
        cudaFree(w->f32);
        cudaFree(w->bx_hi);
        delete w;
        b2m_throw(B2M_ERR_OUT_OF_MEMORY, "weight allocation failed");
      }
      w->seg_bytes[SEG_BX_HI] = hi.size() * 2;
      w->seg_bytes[SEG_BX_LO] = lo.size() * 2;
      B2M_CUDA(cudaMemcpy(w->bx_hi, hi.data(), hi.size() * 2, cudaMemcpyHostToDevice));
      B2M_CUDA(cudaMemcpy(w->bx_lo, lo.data(), lo.size() * 2, cudaMemcpyHostToDevice));
    }
    *out = w;
  });
}

B2M_API b2m_status b2m_weight_prepack_i8(b2m_ctx *ctx, const void *host_b, int32_t dtype, int64_t k, int64_t n,
                                         b2m_weight **out) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(out && host_b && k > 0 && n > 0, B2M_ERR_INVALID_ARGUMENT, "MatMulInteger prepack: bad arguments");
    B2M_REQUIRE(is_i8(dtype), B2M_ERR_INVALID_ARGUMENT, "MatMulInteger prepack: dtype must be uint8 or int8");
    DeviceGuard dg(ctx->device);
    const int64_t kpad = round_up(k, 64), npad = round_up(n, 128);
    std::vector<int8_t> bt((size_t)(npad * kpad), 0);
    std::vector<int32_t> cs((size_t)n, 0);
    const uint8_t *src = static_cast<const uint8_t *>(host_b);
    for (int64_t kk = 0; kk < k; kk++)
      for (int64_t j = 0; j < n; j++) {
        const uint8_t v = src[kk * n + j];
        bt[(size_t)(j * kpad + kk)] = (int8_t)v;
        cs[(size_t)j] += dtype == B2M_INT8 ? (int32_t)(int8_t)v : (int32_t)v;
      }
    b2m_weight *w = new b2m_weight();
    w->ctx = ctx;
    w->kind = W_I8;
    w->k = k;
    w->n = n;
    w->i8.dtype = dtype;
    w->i8.kpad = kpad;
    w->i8.npad = npad;
    // ts8: per (128-column tile, 128-k chunk) eight planes of 128 columns x
    // 16 bytes (k_int8_tc.cu); zero padded to npad x k128.
    const int64_t k128 = round_up(k, 128), nch = k128 / 128;
    std::vector<uint8_t> ts8((size_t)(npad * k128), 0);
    for (int64_t kk = 0; kk < k; kk++) {
      const int64_t ch = kk / 128, pl = (kk % 128) / 16, by = kk % 16;
      for (int64_t j = 0; j < n; j++) {
        const int64_t tile = j / 128, cl = j % 128;
        ts8[(size_t)((((tile * nch + ch) * 8 + pl) * 128 + cl) * 16 + by)] = src[kk * n + j];
      }
    }
    w->i8.k128 = k128;
    try {
      B2M_CUDA(cudaMalloc(&w->i8.bt, bt.size()));
      B2M_CUDA(cudaMalloc(&w->i8.colsum, cs.size() * 4));
      B2M_CUDA(cudaMalloc(&w->i8.ts8, ts8.size()));
      w->seg_bytes[SEG_I8_BT] = bt.size();
      w->seg_bytes[SEG_I8_COLSUM] = cs.size() * 4;
      w->seg_bytes[SEG_I8_TS8] = ts8.size();
      B2M_CUDA(cudaMemcpy(w->i8.bt, bt.data(), bt.size(), cudaMemcpyHostToDevice));
      B2M_CUDA(cudaMemcpy(w->i8.colsum, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
      B2M_CUDA(cudaMemcpy(w->i8.ts8, ts8.data(), ts8.size(), cudaMemcpyHostToDevice));
    } catch (...) {
      cudaFree(w->i8.bt);
      cudaFree(w->i8.colsum);
      cudaFree(w->i8.ts8);
      delete w;
      throw;
    }
    *out = w;
  });
}

B2M_API b2m_status b2m_weight_prepack_nbits(b2m_ctx *ctx, const uint8_t *b_q, const float *scales,
                                            const void *zero_points, int32_t zp_dtype, int64_t k, int64_t n,
                                            int32_t bits, int32_t block_size, b2m_weight **out) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(out && b_q && scales, B2M_ERR_INVALID_ARGUMENT, "MatMulNBits prepack: null argument");
    // Same checks, same order, same error classes as opMatMulNBits (:126-135).
    if (bits != 4) b2m_throw(B2M_ERR_UNSUPPORTED, "MatMulNBits: only bits=4 supported, got " + std::to_string(bits));
    if (k <= 0 || n <= 0 || block_size < 16 || (block_size & (block_size - 1)) != 0)
      b2m_throw(B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: invalid K, N, block_size or input shape");
    B2M_REQUIRE(zp_dtype == 0 || zp_dtype == B2M_UINT8 || zp_dtype == B2M_FLOAT, B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits: invalid zero_points");
    B2M_REQUIRE((zp_dtype == 0) == (zero_points == nullptr), B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits: invalid zero_points");
    DeviceGuard dg(ctx->device);
    const int64_t nb = (k + block_size - 1) / block_size;
    const int64_t blob = block_size / 2;
    const int64_t zs = (nb + 1) / 2;
    const int64_t kp = round_up(nb * block_size, 64);
    const int64_t npad = round_up(n, 128);
    const int64_t row = kp / 2;
    // Fragment-major layout (see k_nbits.cu): record (tile of 16 columns,
    // chunk of 64 k) = 32 lanes x 16 bytes; lane 4g+t holds the words
    // (group 0, col g), (group 0, col g+8), (group 1, col g), (group 1, col g+8),
    // each word = original bytes 2t, 2t+1, 8+2t, 9+2t of that 32-k group.
    const int64_t nchunks = kp / 64;
    std::vector<uint8_t> bq((size_t)(npad * row), 0);
    std::vector<uint8_t> tmp((size_t)row);
    for (int64_t c = 0; c < n; c++) {
      std::fill(tmp.begin(), tmp.end(), 0);
      std::memcpy(tmp.data(), b_q + c * nb * blob, (size_t)(nb * blob));
      const int64_t tile = c / 16;
      const int cc = (int)(c % 16), g = cc % 8, hi = cc / 8;
      for (int64_t G = 0; G < kp / 32; G++) {
        const uint8_t *o = &tmp[(size_t)(G * 16)];
        const int64_t chunk = G / 2;
        const int grp = (int)(G % 2);
        for (int t = 0; t < 4; t++) {
          uint8_t *d = &bq[(size_t)(((tile * nchunks + chunk) * 32 + (g * 4 + t)) * 16 + 4 * (2 * grp + hi))];
          d[0] = o[2 * t];
          d[1] = o[2 * t + 1];
          d[2] = o[8 + 2 * t];
          d[3] = o[9 + 2 * t];
        }
      }
    }
    std::vector<float> sc((size_t)(npad * nb), 0.f);
    std::memcpy(sc.data(), scales, (size_t)(n * nb * 4));
    b2m_weight *w = new b2m_weight();
    w->ctx = ctx;
    w->kind = W_NBITS;
    w->k = k;
    w->n = n;
    NbitsWeight &W = w->nb;
    W.block = block_size;
    W.nblocks = nb;
    {
      bool ok16 = zp_dtype != B2M_FLOAT;
      for (int64_t i = 0; i < n * nb && ok16; i++) {
        const float a = std::fabs(scales[i]);
        ok16 = a == 0.f || (a >= 6.103515625e-05f && a <= 65504.f);
      }
      W.f16_scales = ok16;
    }
    std::vector<__half> srec;
    if (W.f16_scales && block_size >= 32) {
      const int64_t ntile = npad / 16;
      srec.assign((size_t)(ntile * nchunks * 8 * 8), __float2half_rn(0.f));
      for (int64_t tl = 0; tl < ntile; tl++)
        for (int64_t ch = 0; ch < nchunks; ch++)
          for (int g = 0; g < 8; g++)
            for (int grp = 0; grp < 2; grp++)
              for (int hi = 0; hi < 2; hi++) {
                const int64_t col = tl * 16 + g + 8 * hi;
                const int64_t blk = (ch * 64 + grp * 32) / block_size;
                float sv = 0.f, zv = 8.f;
                if (col < n && blk < nb) {
                  sv = scales[col * nb + blk];
                  if (zp_dtype == B2M_UINT8) {
                    const uint8_t zb = static_cast<const uint8_t *>(zero_points)[col * zs + blk / 2];
                    zv = (float)((blk & 1) ? (zb >> 4) : (zb & 15));
                  }
                }
                const size_t o = (size_t)(((tl * nchunks + ch) * 8 + g) * 8 + grp * 4 + hi * 2);
                srec[o] = __float2half_rn(sv);
                srec[o + 1] = __float2half_rn(1024.f + zv);
              }
    }
    // TMEM-operand prefill layout (k_nbits_ts.cu), same eligibility.
    std::vector<uint8_t> tsq;
    std::vector<uint32_t> tss;
    if (W.f16_scales && block_size >= 32) {
      static const int pos[8] = {0, 16, 4, 20, 8, 24, 12, 28};
      tsq.assign((size_t)(npad * kp / 2), 0);
      tss.assign((size_t)(npad * nchunks * 2), 0u);
      for (int64_t c = 0; c < npad; c++) {
        const int64_t tile = c / 128, cl = c % 128;
        const uint8_t *src = c < n ? b_q + c * nb * blob : nullptr;
        for (int64_t ch = 0; ch < nchunks; ch++) {
          for (int j = 0; j < 8; j++) {
            uint32_t word = 0;
            for (int i = 0; i < 8; i++) {
              const int64_t kk = ch * 64 + 8 * j + i;
              if (src && kk < nb * block_size) {
                const uint8_t byte = src[kk / 2];
                word |= (uint32_t)((kk & 1) ? (byte >> 4) : (byte & 15)) << pos[i];
              }
            }
            const size_t off = ((size_t)((tile * nchunks + ch) * 2 + j / 4) * 128 + (size_t)cl) * 16 + (j % 4) * 4;
            std::memcpy(&tsq[off], &word, 4);
          }
          for (int g = 0; g < 2; g++) {
            const int64_t blk = (ch * 64 + g * 32) / block_size;
            float sv = 0.f, zv = 8.f;
            if (c < n && blk < nb) {
              sv = scales[c * nb + blk];
              if (zp_dtype == B2M_UINT8) {
                const uint8_t zb = static_cast<const uint8_t *>(zero_points)[c * zs + blk / 2];
                zv = (float)((blk & 1) ? (zb >> 4) : (zb & 15));
              }
            }
            const __half hs = __float2half_rn(sv), hz = __float2half_rn(1024.f + zv);
            uint16_t us, uz;
            std::memcpy(&us, &hs, 2);
            std::memcpy(&uz, &hz, 2);
            tss[((size_t)(tile * nchunks + ch) * 128 + (size_t)cl) * 2 + g] = (uint32_t)us | ((uint32_t)uz << 16);
          }
        }
      }
    }
    W.zstride = zs;
    W.kp = kp;
    W.npad = npad;
    try {
      B2M_CUDA(cudaMalloc(&W.bq, bq.size()));
      w->seg_bytes[SEG_NB_BQ] = bq.size();
      B2M_CUDA(cudaMemcpy(W.bq, bq.data(), bq.size(), cudaMemcpyHostToDevice));
      B2M_CUDA(cudaMalloc(&W.scales, sc.size() * 4));
      w->seg_bytes[SEG_NB_SCALES] = sc.size() * 4;
      B2M_CUDA(cudaMemcpy(W.scales, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice));
      if (!srec.empty()) {
        B2M_CUDA(cudaMalloc(&W.srec, srec.size() * sizeof(__half)));
        w->seg_bytes[SEG_NB_SREC] = srec.size() * sizeof(__half);
        B2M_CUDA(cudaMemcpy(W.srec, srec.data(), srec.size() * sizeof(__half), cudaMemcpyHostToDevice));
      }
      if (!tsq.empty()) {
        B2M_CUDA(cudaMalloc(&W.tsq, tsq.size()));
        w->seg_bytes[SEG_NB_TSQ] = tsq.size();
        B2M_CUDA(cudaMemcpy(W.tsq, tsq.data(), tsq.size(), cudaMemcpyHostToDevice));
        B2M_CUDA(cudaMalloc(&W.tss, tss.size() * 4));
        w->seg_bytes[SEG_NB_TSS] = tss.size() * 4;
        B2M_CUDA(cudaMemcpy(W.tss, tss.data(), tss.size() * 4, cudaMemcpyHostToDevice));
      }
      if (zp_dtype == B2M_UINT8) {
        std::vector<uint8_t> z((size_t)(npad * zs), 0);
        std::memcpy(z.data(), zero_points, (size_t)(n * zs));
        W.zp_kind = 1;
        B2M_CUDA(cudaMalloc(&W.zp_u8, z.size()));
        w->seg_bytes[SEG_NB_ZP_U8] = z.size();
        B2M_CUDA(cudaMemcpy(W.zp_u8, z.data(), z.size(), cudaMemcpyHostToDevice));
      } else if (zp_dtype == B2M_FLOAT) {
        std::vector<float> z((size_t)(npad * nb), 0.f);
        std::memcpy(z.data(), zero_points, (size_t)(n * nb * 4));
        W.zp_kind = 2;
        B2M_CUDA(cudaMalloc(&W.zp_f32, z.size() * 4));
        w->seg_bytes[SEG_NB_ZP_F32] = z.size() * 4;
        B2M_CUDA(cudaMemcpy(W.zp_f32, z.data(), z.size() * 4, cudaMemcpyHostToDevice));
      }
      nbits_build_drec(W, ctx->stream);
      B2M_CUDA(cudaStreamSynchronize(ctx->stream));
    } catch (...) {
      cudaFree(W.drec);
      cudaFree(W.bq);
      cudaFree(W.scales);
      cudaFree(W.zp_u8);
      cudaFree(W.zp_f32);
      cudaFree(W.srec);
      cudaFree(W.tsq);
      cudaFree(W.tss);
      delete w;
      throw;
    }
    *out = w;
  });
}

B2M_API b2m_status b2m_weight_set_next(b2m_weight *w, const b2m_weight *next) {
  return guarded([&] {
    B2M_REQUIRE(w, B2M_ERR_INVALID_ARGUMENT, "null weight");
    B2M_REQUIRE(!next || next->ctx == w->ctx, B2M_ERR_INVALID_ARGUMENT,
                "weight set_next: both weights must belong to one context");
    if (next)
      w->ctx->next_of[w] = next;
    else
      w->ctx->next_of.erase(w);
  });
}

B2M_API b2m_status b2m_weight_free(b2m_weight *w) {
  return guarded([&] {
    if (!w) return;
    DeviceGuard dg(w->ctx->device);
    cudaStreamSynchronize(w->ctx->stream);
    // No later launch may prefetch this weight, nor prefetch for it.
    auto &nx = w->ctx->next_of;
    for (auto it = nx.begin(); it != nx.end();) it = (it->first == w || it->second == w) ? nx.erase(it) : std::next(it);
    cudaFree(w->f32);
    cudaFree(w->bx_hi);
    cudaFree(w->bx_lo);
    cudaFree(w->i8.bt);
    cudaFree(w->i8.colsum);
    cudaFree(w->i8.ts8);
    cudaFree(w->nb.bq);
    cudaFree(w->nb.scales);
    cudaFree(w->nb.zp_u8);
    cudaFree(w->nb.zp_f32);
    cudaFree(w->nb.wdeq);
    cudaFree(w->nb.px_hi);
    cudaFree(w->nb.px_lo);
    cudaFree(w->nb.srec);
    cudaFree(w->nb.tsq);
    cudaFree(w->nb.tss);
    cudaFree(w->nb.drec);
    delete w;
  });
}

}  // extern "C"

namespace {

// Serialised packed weight: a fixed header, the scalar fields, the byte size
// of every device buffer, then the buffers in segment order.
constexpr uint32_t WEIGHT_MAGIC = 0x574d3242u;  // "B2MW"
constexpr uint32_t WEIGHT_FORMAT = 1;
constexpr int WEIGHT_FIELDS = 13;

void **segment_slot(b2m_weight *w, int id) {
  switch (id) {
    case SEG_F32: return reinterpret_cast<void **>(&w->f32);
    case SEG_BX_HI: return reinterpret_cast<void **>(&w->bx_hi);
    case SEG_BX_LO: return reinterpret_cast<void **>(&w->bx_lo);
    case SEG_I8_BT: return reinterpret_cast<void **>(&w->i8.bt);
    case SEG_I8_COLSUM: return reinterpret_cast<void **>(&w->i8.colsum);
    case SEG_I8_TS8: return reinterpret_cast<void **>(&w->i8.ts8);
    case SEG_NB_BQ: return reinterpret_cast<void **>(&w->nb.bq);
    case SEG_NB_SCALES: return reinterpret_cast<void **>(&w->nb.scales);
    case SEG_NB_ZP_U8: return reinterpret_cast<void **>(&w->nb.zp_u8);
    case SEG_NB_ZP_F32: return reinterpret_cast<void **>(&w->nb.zp_f32);
    case SEG_NB_SREC: return reinterpret_cast<void **>(&w->nb.srec);
    case SEG_NB_TSQ: return reinterpret_cast<void **>(&w->nb.tsq);
    default: return reinterpret_cast<void **>(&w->nb.tss);
  }
}

void weight_fields(const b2m_weight *w, int64_t (&f)[WEIGHT_FIELDS]) {
  const int64_t v[WEIGHT_FIELDS] = {w->k, w->n, w->i8.dtype, w->i8.kpad, w->i8.npad, w->i8.k128, w->nb.zp_kind,
                                    w->nb.block, w->nb.nblocks, w->nb.zstride, w->nb.kp, w->nb.npad,
                                    w->nb.f16_scales ? 1 : 0};
  for (int i = 0; i < WEIGHT_FIELDS; i++) f[i] = v[i];
}

size_t weight_blob_bytes(const b2m_weight *w) {
  size_t n = 4 * sizeof(uint32_t) + WEIGHT_FIELDS * sizeof(int64_t) + SEG_COUNT * sizeof(uint64_t);
  for (int i = 0; i < SEG_COUNT; i++) n += w->seg_bytes[i];
  return n;
}

}  // namespace

extern "C" {

B2M_API b2m_status b2m_weight_export(const b2m_weight *w, void *buf, size_t capacity, size_t *needed) {
  return guarded([&] {
    B2M_REQUIRE(w && needed, B2M_ERR_INVALID_ARGUMENT, "weight export: null argument");
    const size_t total = weight_blob_bytes(w);
    *needed = total;
    if (!buf) return;
    B2M_REQUIRE(capacity >= total, B2M_ERR_INVALID_ARGUMENT, "weight export: buffer too small");
    DeviceGuard dg(w->ctx->device);
    B2M_CUDA(cudaStreamSynchronize(w->ctx->stream));
    uint8_t *p = static_cast<uint8_t *>(buf);
    const uint32_t hdr[4] = {WEIGHT_MAGIC, WEIGHT_FORMAT, (uint32_t)B2M_ABI_VERSION, (uint32_t)w->kind};
    std::memcpy(p, hdr, sizeof(hdr));
    p += sizeof(hdr);
    int64_t f[WEIGHT_FIELDS];
    weight_fields(w, f);
    std::memcpy(p, f, sizeof(f));
    p += sizeof(f);
    for (int i = 0; i < SEG_COUNT; i++) {
      const uint64_t b = w->seg_bytes[i];
      std::memcpy(p, &b, sizeof(b));
      p += sizeof(b);
    }
    for (int i = 0; i < SEG_COUNT; i++) {
      if (!w->seg_bytes[i]) continue;
      void *dev = *segment_slot(const_cast<b2m_weight *>(w), i);
      B2M_REQUIRE(dev, B2M_ERR_CUDA, "weight export: missing device buffer");
      B2M_CUDA(cudaMemcpy(p, dev, w->seg_bytes[i], cudaMemcpyDeviceToHost));
      p += w->seg_bytes[i];
    }
  });
}

B2M_API b2m_status b2m_weight_import(b2m_ctx *ctx, const void *buf, size_t size, b2m_weight **out) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(buf && out, B2M_ERR_INVALID_ARGUMENT, "weight import: null argument");
    const size_t head = 4 * sizeof(uint32_t) + WEIGHT_FIELDS * sizeof(int64_t) + SEG_COUNT * sizeof(uint64_t);
    B2M_REQUIRE(size >= head, B2M_ERR_INVALID_ARGUMENT, "weight import: truncated header");
    const uint8_t *p = static_cast<const uint8_t *>(buf);
    uint32_t hdr[4];
    std::memcpy(hdr, p, sizeof(hdr));
    p += sizeof(hdr);
    B2M_REQUIRE(hdr[0] == WEIGHT_MAGIC && hdr[1] == WEIGHT_FORMAT, B2M_ERR_INVALID_ARGUMENT,
                "weight import: not a packed-weight blob");
    B2M_REQUIRE(hdr[2] == (uint32_t)B2M_ABI_VERSION, B2M_ERR_UNSUPPORTED,
                "weight import: blob written by another library version");
    B2M_REQUIRE(hdr[3] == W_F32 || hdr[3] == W_I8 || hdr[3] == W_NBITS, B2M_ERR_INVALID_ARGUMENT,
                "weight import: unknown weight kind");
    int64_t f[WEIGHT_FIELDS];
    std::memcpy(f, p, sizeof(f));
    p += sizeof(f);
    uint64_t segb[SEG_COUNT];
    std::memcpy(segb, p, sizeof(segb));
    p += sizeof(segb);
    size_t total = head;
    for (int i = 0; i < SEG_COUNT; i++) {
      B2M_REQUIRE(segb[i] <= size, B2M_ERR_INVALID_ARGUMENT, "weight import: bad segment size");
      total += segb[i];
    }
    B2M_REQUIRE(total == size, B2M_ERR_INVALID_ARGUMENT, "weight import: size mismatch");
    DeviceGuard dg(ctx->device);
    b2m_weight *w = new b2m_weight();
    w->ctx = ctx;
    w->kind = (int)hdr[3];
    w->k = f[0];
    w->n = f[1];
    w->i8.dtype = (int32_t)f[2];
    w->i8.kpad = f[3];
    w->i8.npad = f[4];
    w->i8.k128 = f[5];
    w->nb.zp_kind = (int)f[6];
    w->nb.block = (int)f[7];
    w->nb.nblocks = f[8];
    w->nb.zstride = f[9];
    w->nb.kp = f[10];
    w->nb.npad = f[11];
    w->nb.f16_scales = f[12] != 0;
    try {
      for (int i = 0; i < SEG_COUNT; i++) {
        if (!segb[i]) continue;
        void **slot = segment_slot(w, i);
        B2M_CUDA(cudaMalloc(slot, segb[i]));
        w->seg_bytes[i] = segb[i];
        B2M_CUDA(cudaMemcpy(*slot, p, segb[i], cudaMemcpyHostToDevice));
        p += segb[i];
      }
      if (w->kind == W_NBITS) {  // the decode records are derived, not stored
        nbits_build_drec(w->nb, ctx->stream);
        B2M_CUDA(cudaStreamSynchronize(ctx->stream));
      }
    } catch (...) {
      cudaFree(w->nb.drec);
      for (int i = 0; i < SEG_COUNT; i++) cudaFree(*segment_slot(w, i));
      delete w;
      throw;
    }
    *out = w;
  });
}

B2M_API b2m_status b2m_weight_info(const b2m_weight *w, int64_t *k, int64_t *n) {
  return guarded([&] {
    B2M_REQUIRE(w, B2M_ERR_INVALID_ARGUMENT, "null weight");
    if (k) *k = w->k;
    if (n) *n = w->n;
  });
}

// ---- operators ------------------------------------------------------------

B2M_API b2m_status b2m_matmul_f32(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b,
                                  const b2m_weight *b_packed, int32_t mode, b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    matmul_f32_impl(ctx, a, b, b_packed, mode, y);
  });
}

B2M_API b2m_status b2m_gemm_f32(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b,
                                const b2m_weight *b_packed, const b2m_tensor *c, float alpha, float beta,
                                int32_t trans_a, int32_t trans_b, int32_t mode, b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    gemm_f32_impl(ctx, a, b, b_packed, c, alpha, beta, trans_a, trans_b, mode, y);
  });
}

B2M_API b2m_status b2m_matmul_integer(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b,
                                      const b2m_weight *b_packed, const b2m_tensor *a_zp, const b2m_tensor *b_zp,
                                      b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    integer_impl(ctx, a, b, b_packed, a_zp, b_zp, false, 0.0, 0, 0, 0, y);
  });
}

B2M_API b2m_status b2m_qlinear_matmul(b2m_ctx *ctx, const b2m_tensor *a, float a_scale, const b2m_tensor *a_zp,
                                      const b2m_tensor *b, const b2m_weight *b_packed, float b_scale,
                                      const b2m_tensor *b_zp, float y_scale, int32_t y_zp, int32_t lo, int32_t hi,
                                      b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    // Requant multiplier exactly as the reference: f32(aS*bS), then f32(/yS),
    // each step rounded to float32 (onnx_qlinear_ops.dart:95-99).
    float f = (float)((double)a_scale * (double)b_scale);
    f = (float)((double)f / (double)y_scale);
    integer_impl(ctx, a, b, b_packed, a_zp, b_zp, true, (double)f, y_zp, lo, hi, y);
  });
}

B2M_API b2m_status b2m_matmul_nbits(b2m_ctx *ctx, const b2m_tensor *a, const b2m_weight *w, const b2m_tensor *bias,
                                    int32_t mode, b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    B2M_REQUIRE(w && w->kind == W_NBITS, B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: weight is not a MatMulNBits weight");
    require_float(a, "MatMulNBits A");
    if (a->rank < 1 || a->shape[a->rank - 1] != w->k)
      b2m_throw(B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: invalid K, N, block_size or input shape");
    if (bias && (bias->dtype != B2M_FLOAT || bias->rank != 1 || bias->numel != w->n))
      b2m_throw(B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: bias must be floating point [N]");
    const int64_t m = a->numel / w->k;
    std::vector<int64_t> oshape(a->shape, a->shape + a->rank - 1);
    oshape.push_back(w->n);
    check_cancel(ctx);
    b2m_tensor *out = prepare_output(ctx, y, B2M_FLOAT, oshape);
    Scratch sc(ctx, nbits_scratch_bytes(w, m, mode));
    OpTimer timer(ctx);
    nbits_run(ctx, sc, static_cast<const float *>(a->data), m, w,
              bias ? static_cast<const float *>(bias->data) : nullptr, mode, static_cast<float *>(out->data));
    timer.done();
  });
}

B2M_API b2m_status b2m_matmul_nbits_dev(b2m_ctx *ctx, const float *a, int64_t m, const b2m_weight *w,
                                        const float *bias, int32_t mode, float *y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    B2M_REQUIRE(m >= 0 && (a || m == 0) && (y || m == 0), B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: bad pointers");
    check_cancel(ctx);
    B2M_REQUIRE(w && w->kind == W_NBITS, B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: weight is not a MatMulNBits weight");
    Scratch sc(ctx, nbits_scratch_bytes(w, m, mode));
    OpTimer timer(ctx);
    nbits_run(ctx, sc, a, m, w, bias, mode, y);
    timer.done();
  });
}

static int32_t nbits_route(const b2m_weight *w, int64_t m, int32_t mode) {
  if (mode == B2M_MODE_FAST) {
    if (nbits_use_smallm(w->nb, m, w->k, w->n)) return B2M_ROUTE_GEMV;
    if (w->nb.tsq && nbits_tc_supported(w->nb, m, w->k, w->n)) return B2M_ROUTE_TC_F16;
    return B2M_ROUTE_OTHER;
  }
  if (mode == B2M_MODE_PRECISE && nbits_precise_gemv(w->nb, m)) return B2M_ROUTE_GEMV;
  return B2M_ROUTE_OTHER;
}

B2M_API b2m_status b2m_matmul_nbits_route(b2m_ctx *ctx, const b2m_weight *w, int64_t m, int32_t mode,
                                          int32_t *route) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(w && w->kind == W_NBITS && route && m >= 0, B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits route: bad arguments");
    *route = m == 0 ? B2M_ROUTE_OTHER : nbits_route(w, m, mode);
  });
}

B2M_API b2m_status b2m_matmul_nbits_f16_dev(b2m_ctx *ctx, const uint16_t *a16, int64_t m, const b2m_weight *w,
                                            const float *bias, float *y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    B2M_REQUIRE(w && w->kind == W_NBITS, B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: weight is not a MatMulNBits weight");
    B2M_REQUIRE(m >= 0 && (m == 0 || (a16 && y)), B2M_ERR_INVALID_ARGUMENT, "MatMulNBits f16: bad pointers");
    check_cancel(ctx);
    if (m == 0) return;
    B2M_REQUIRE(w->k % 8 == 0 && (reinterpret_cast<uintptr_t>(a16) & 15) == 0 &&
                    nbits_route(w, m, B2M_MODE_FAST) == B2M_ROUTE_TC_F16,
                B2M_ERR_UNSUPPORTED, "MatMulNBits f16: the call's route does not take f16 activations");
    OpTimer timer(ctx);
    NbitsArgs p;
    p.A = nullptr;
    p.w = &w->nb;
    p.bias = bias;
    p.Y = y;
    p.M = m;
    p.K = w->k;
    p.N = w->n;
    p.dev_err = ctx->dev_err;
    nbits_prefetch_plan(ctx, w, m, B2M_MODE_FAST, p);
    launch_nbits_ts(p, reinterpret_cast<const __half *>(a16), w->k, ctx->stream);
    timer.done();
  });
}

B2M_API b2m_status b2m_matmul_nbits_swiglu_dev(b2m_ctx *ctx, const float *a, const uint16_t *a16, int64_t m,
                                               const b2m_weight *w, int32_t mode, float *act, uint16_t *act16) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    B2M_REQUIRE(w && w->kind == W_NBITS, B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: weight is not a MatMulNBits weight");
    B2M_REQUIRE(mode == B2M_MODE_EXACT || mode == B2M_MODE_FAST || mode == B2M_MODE_PRECISE,
                B2M_ERR_INVALID_ARGUMENT, "MatMulNBits SwiGLU: bad mode");
    B2M_REQUIRE(w->n % 128 == 0, B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits SwiGLU: N must be a multiple of 128 (tile-interleaved gate / up rows)");
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    B2M_REQUIRE(m >= 0 && (m == 0 || ((a || a16) && (act || act16))) && al(act) && al(act16),
                B2M_ERR_INVALID_ARGUMENT, "MatMulNBits SwiGLU: bad pointers (act / act16 16-byte aligned)");
    check_cancel(ctx);
    if (m == 0) return;
    const int64_t I = w->n / 2;
    OpTimer timer(ctx);
    const bool tc = mode == B2M_MODE_FAST && nbits_route(w, m, mode) == B2M_ROUTE_TC_F16;
    if (tc && (a16 ? (w->k % 8 == 0 && al(a16)) : true)) {
      NbitsArgs p;
      p.A = a;
      p.w = &w->nb;
      p.bias = nullptr;
      p.Y = nullptr;
      p.M = m;
      p.K = w->k;
      p.N = w->n;
      p.dev_err = ctx->dev_err;
      nbits_prefetch_plan(ctx, w, m, mode, p);
      const int64_t K8 = nbits_tc_k8(w->k);
      Scratch sc(ctx, a16 ? 0 : (size_t)(m * K8 * 2) + 256);
      const __half *x16 = reinterpret_cast<const __half *>(a16);
      if (!a16) {
        __half *c16 = static_cast<__half *>(sc.take((size_t)(m * K8 * 2)));
        b2m::launch_f32_to_f16(a, c16, m, w->k, K8, 0, ctx->stream);
        x16 = c16;
      }
      launch_nbits_ts(p, x16, a16 ? w->k : K8, ctx->stream, act, reinterpret_cast<__half *>(act16));
    } else {
      B2M_REQUIRE(a, B2M_ERR_UNSUPPORTED, "MatMulNBits SwiGLU: this call's route takes fp32 activations (a is null)");
      const size_t ybytes = (size_t)(m * w->n * 4);
      Scratch sc(ctx, ybytes + 256 + nbits_scratch_bytes(w, m, mode));
      float *y = static_cast<float *>(sc.take(ybytes));
      nbits_run(ctx, sc, a, m, w, nullptr, mode, y);
      launch_silu_mul_tiles(y, m, I, act, reinterpret_cast<__half *>(act16), ctx->stream);
    }
    timer.done();
  });
}

B2M_API b2m_status b2m_matmul_nbits_host(b2m_ctx *ctx, const float *a_host, int64_t m, const b2m_weight *w,
                                         const float *bias_host, int32_t mode, float *y_host) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    B2M_REQUIRE(w && w->kind == W_NBITS, B2M_ERR_INVALID_ARGUMENT, "MatMulNBits: weight is not a MatMulNBits weight");
    B2M_REQUIRE(m >= 0 && (a_host || m == 0) && (y_host || m == 0), B2M_ERR_INVALID_ARGUMENT,
                "MatMulNBits: bad host pointers");
    check_cancel(ctx);
    if (m == 0) return;
    const size_t abytes = (size_t)(m * w->k * 4), ybytes = (size_t)(m * w->n * 4), bbytes = (size_t)(w->n * 4);
    Scratch sc(ctx, abytes + ybytes + bbytes + 1024 + nbits_scratch_bytes(w, m, mode));
    float *da = static_cast<float *>(sc.take(abytes));
    // The decode GEMV stores Y (one 64-byte segment per CTA and row) straight
    // into a pinned y_host: no device-to-host copy to queue and wait for.
    // Other routes, and pageable y_host, go through device memory.
    const bool gemv = mode == B2M_MODE_FAST ? nbits_use_smallm(w->nb, m, w->k, w->n)
                                            : mode == B2M_MODE_PRECISE && nbits_precise_gemv(w->nb, m);
    float *dy = gemv ? static_cast<float *>(mapped_host_ptr(y_host)) : nullptr;
    const bool direct_y = dy != nullptr;
    if (!direct_y) dy = static_cast<float *>(sc.take(ybytes));
    float *db = bias_host ? static_cast<float *>(sc.take(bbytes)) : nullptr;
    B2M_CUDA(cudaMemcpyAsync(da, a_host, abytes, cudaMemcpyHostToDevice, ctx->stream));
    if (db) B2M_CUDA(cudaMemcpyAsync(db, bias_host, bbytes, cudaMemcpyHostToDevice, ctx->stream));
    OpTimer timer(ctx);
    nbits_run(ctx, sc, da, m, w, db, mode, dy);
    timer.done();
    if (!direct_y) B2M_CUDA(cudaMemcpyAsync(y_host, dy, ybytes, cudaMemcpyDeviceToHost, ctx->stream));
    B2M_CUDA(cudaStreamSynchronize(ctx->stream));
    raise_device_error(ctx);
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Transformer glue (device pointers)
// ---------------------------------------------------------------------------

B2M_API b2m_status b2m_rmsnorm_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma, float *y,
                                   float *sum_out, int64_t rows, int64_t d, double eps) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && d > 0 && d <= (1 << 24) && (rows == 0 || (x && gamma && y)), B2M_ERR_INVALID_ARGUMENT,
                "RMSNorm: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_rmsnorm(x, skip, gamma, y, sum_out, rows, (int)d, eps, std::max<int64_t>(rows, 1), 0, ctx->stream);
  });
}

B2M_API b2m_status b2m_rmsnorm_f16_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma, float *y,
                                       float *sum_out, uint16_t *y16, int64_t rows, int64_t d, double eps) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && d > 0 && d % 8 == 0 && d <= (1 << 24) && (rows == 0 || (x && gamma && y16)),
                B2M_ERR_INVALID_ARGUMENT, "RMSNorm f16: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_rmsnorm(x, skip, gamma, y, sum_out, rows, (int)d, eps, std::max<int64_t>(rows, 1), 0, ctx->stream, 0,
                   reinterpret_cast<__half *>(y16));
  });
}

B2M_API b2m_status b2m_rmsnorm_heads_dev(b2m_ctx *ctx, const float *x, const float *gamma, float *y, int64_t tokens,
                                         int64_t heads, int64_t head_dim, int64_t token_stride, double eps) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(tokens >= 0 && heads > 0 && head_dim > 0 && head_dim <= (1 << 24) &&
                    token_stride >= heads * head_dim && (tokens == 0 || (x && gamma && y)),
                B2M_ERR_INVALID_ARGUMENT, "RMSNorm heads: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_rmsnorm(x, nullptr, gamma, y, nullptr, tokens * heads, (int)head_dim, eps, heads, token_stride,
                   ctx->stream);
  });
}

B2M_API b2m_status b2m_rmsnorm_head_rows_dev(b2m_ctx *ctx, const float *x, const float *gamma_rows, float *y,
                                             int64_t tokens, int64_t heads, int64_t head_dim, int64_t token_stride,
                                             double eps) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(tokens >= 0 && heads > 0 && head_dim > 0 && head_dim <= (1 << 24) &&
                    token_stride >= heads * head_dim && (tokens == 0 || (x && gamma_rows && y)),
                B2M_ERR_INVALID_ARGUMENT, "RMSNorm head rows: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_rmsnorm(x, nullptr, gamma_rows, y, nullptr, tokens * heads, (int)head_dim, eps, heads, token_stride,
                   ctx->stream, head_dim);
  });
}

B2M_API b2m_status b2m_layernorm_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma,
                                     const float *beta, float *y, float *sum_out, int64_t rows, int64_t d,
                                     double eps) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && d > 0 && d <= (1 << 24) && (rows == 0 || (x && gamma && y)), B2M_ERR_INVALID_ARGUMENT,
                "LayerNormalization: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_layernorm(x, skip, gamma, beta, y, sum_out, rows, (int)d, eps, ctx->stream);
  });
}

B2M_API b2m_status b2m_layernorm_split_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma,
                                           const float *beta, float *y, float *sum_out, uint16_t *y_planes,
                                           int64_t rows, int64_t d, double eps) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && d > 0 && d % 64 == 0 && d <= (1 << 24) && (rows == 0 || (x && gamma && y && y_planes)),
                B2M_ERR_INVALID_ARGUMENT, "LayerNormalization split: bad arguments");
    DeviceGuard dg(ctx->device);
    __nv_bfloat16 *p0 = reinterpret_cast<__nv_bfloat16 *>(y_planes);
    launch_layernorm(x, skip, gamma, beta, y, sum_out, rows, (int)d, eps, ctx->stream, p0, p0 + rows * d);
  });
}

B2M_API b2m_status b2m_silu_mul_dev(b2m_ctx *ctx, const float *gate, const float *up, int64_t gate_rs,
                                    int64_t up_rs, float *y, int64_t rows, int64_t d) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && d >= 0 && gate_rs >= d && up_rs >= d && (rows * d == 0 || (gate && up && y)),
                B2M_ERR_INVALID_ARGUMENT, "SiLU*Mul: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_silu_mul(gate, up, gate_rs, up_rs, y, rows, d, ctx->stream);
  });
}

B2M_API b2m_status b2m_silu_mul_f16_dev(b2m_ctx *ctx, const float *gate, const float *up, int64_t gate_rs,
                                        int64_t up_rs, float *y, uint16_t *y16, int64_t rows, int64_t d) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && d >= 0 && d % 8 == 0 && gate_rs >= d && up_rs >= d &&
                    (rows * d == 0 || (gate && up && y && y16)),
                B2M_ERR_INVALID_ARGUMENT, "SiLU*Mul f16: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_silu_mul(gate, up, gate_rs, up_rs, y, rows, d, ctx->stream, reinterpret_cast<__half *>(y16));
  });
}

B2M_API b2m_status b2m_gelu_dev(b2m_ctx *ctx, const float *x, float *y, int64_t n) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(n >= 0 && (n == 0 || (x && y)), B2M_ERR_INVALID_ARGUMENT, "Gelu: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_gelu(x, y, n, ctx->stream);
  });
}

B2M_API b2m_status b2m_gelu_split_dev(b2m_ctx *ctx, const float *x, float *y, uint16_t *y_planes, int64_t rows,
                                      int64_t d) {
  return guarded([&] {
    check_ctx(ctx);
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    B2M_REQUIRE(rows >= 0 && d > 0 && d % 64 == 0 &&
                    (rows == 0 || (x && y_planes && al(x) && al(y) && al(y_planes))),
                B2M_ERR_INVALID_ARGUMENT, "Gelu split: bad arguments");
    DeviceGuard dg(ctx->device);
    __nv_bfloat16 *p0 = reinterpret_cast<__nv_bfloat16 *>(y_planes);
    launch_gelu_split(x, y, p0, p0 + rows * d, rows * d, ctx->stream);
  });
}

B2M_API b2m_status b2m_gemm_f32_split_dev(b2m_ctx *ctx, const uint16_t *a_planes, int64_t m, const b2m_weight *w,
                                          const float *bias, float *y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    B2M_REQUIRE(w && w->kind == W_F32 && w->bx_hi, B2M_ERR_INVALID_ARGUMENT,
                "Gemm split: the weight is not an fp32 weight with FAST planes");
    B2M_REQUIRE(m >= 0 && (m == 0 || (a_planes && y)), B2M_ERR_INVALID_ARGUMENT, "Gemm split: bad pointers");
    check_cancel(ctx);
    if (m == 0) return;
    F32GemmArgs p;
    p.A = nullptr;
    p.B = w->f32;
    p.Y = y;
    p.M = m;
    p.N = w->n;
    p.K = w->k;
    p.sa_m = w->k;
    p.sa_k = 1;
    p.sb_k = w->n;
    p.sb_n = 1;
    p.ldy = w->n;
    p.m_eff = m;
    p.tile_w = w->n;
    p.batch = 1;
    p.epi = EPI_GEMM;
    if (bias) {
      p.C = bias;
      p.c_rs = 0;
      p.c_cs = 1;
    }
    p.dev_err = ctx->dev_err;
    B2M_REQUIRE(f32_tc_shape_ok(p), B2M_ERR_UNSUPPORTED, "Gemm split: shape not supported by the FAST GEMM");
    OpTimer timer(ctx);
    launch_f32_tc_planes(p, w->bx_hi, w->bx_lo, w->n, a_planes, 0, 0, ctx->stream);
    timer.done();
  });
}

B2M_API b2m_status b2m_add_dev(b2m_ctx *ctx, const float *a, const float *b, float *y, int64_t rows, int64_t d,
                               int32_t b_broadcast) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && d >= 0 && (rows * d == 0 || (a && b && y)), B2M_ERR_INVALID_ARGUMENT,
                "Add: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_add(a, b, y, rows, d, b_broadcast ? 1 : 0, ctx->stream);
  });
}

B2M_API b2m_status b2m_gather_rows_dev(b2m_ctx *ctx, const float *table, const int64_t *ids, float *y,
                                       int64_t rows, int64_t v, int64_t d) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && v > 0 && d > 0 && (rows == 0 || (table && ids && y)), B2M_ERR_INVALID_ARGUMENT,
                "Gather: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_gather_rows(table, ids, y, rows, v, d, ctx->dev_err, ctx->stream);
  });
}

B2M_API b2m_status b2m_argmax_dev(b2m_ctx *ctx, const float *x, int64_t *out, int64_t rows, int64_t v) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(rows >= 0 && v > 0 && (rows == 0 || (x && out)), B2M_ERR_INVALID_ARGUMENT, "ArgMax: bad arguments");
    DeviceGuard dg(ctx->device);
    if (rows == 0) return;
    const size_t np = (size_t)(rows * argmax_chunks(rows, v));
    Scratch sc(ctx, np * 12 + 512);
    float *pv = static_cast<float *>(sc.take(np * 4));
    int64_t *pi = static_cast<int64_t *>(sc.take(np * 8));
    launch_argmax(x, out, rows, v, pv, pi, ctx->stream);
  });
}

static b2m_status gqa_impl(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                           int64_t kv_rs, float *k_cache, float *v_cache, const int32_t *past,
                           const float *cos_cache, const float *sin_cache, int32_t rotary_half, int32_t rotary_dim,
                           int32_t interleaved, float *out, int32_t b, int32_t s, int32_t h, int32_t kvh,
                           int32_t head_dim, int32_t cap, float scale, uint16_t *out16,
                           const float *qk_gain = nullptr, double qk_eps = 0.0) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(b >= 0 && s >= 0 && h > 0 && kvh > 0 && h % kvh == 0 && head_dim > 0 && head_dim <= 256 && cap > 0,
                B2M_ERR_INVALID_ARGUMENT, "GroupQueryAttention: bad shape arguments");
    B2M_REQUIRE(q_rs >= (int64_t)h * head_dim && kv_rs >= (int64_t)kvh * head_dim, B2M_ERR_INVALID_ARGUMENT,
                "GroupQueryAttention: row strides too small");
    B2M_REQUIRE((int64_t)b * s == 0 || (q && k && v && k_cache && v_cache && past && (out || out16)),
                B2M_ERR_INVALID_ARGUMENT, "GroupQueryAttention: null pointer");
    B2M_REQUIRE(!out16 || ((int64_t)h * head_dim) % 8 == 0, B2M_ERR_INVALID_ARGUMENT,
                "GroupQueryAttention f16: h * head_dim must be a multiple of 8");
    const bool rot = cos_cache != nullptr;
    B2M_REQUIRE(!rot || (sin_cache && rotary_half > 0 && rotary_dim > 0 && rotary_dim <= head_dim &&
                         rotary_dim % 2 == 0 && rotary_dim / 2 <= rotary_half),
                B2M_ERR_INVALID_ARGUMENT, "GroupQueryAttention: bad rotary arguments");
    DeviceGuard dg(ctx->device);
    if ((int64_t)b * s == 0) return;
    const float sc = scale > 0.f ? scale : 1.f / std::sqrt((float)head_dim);
    const int nsplit = ctx->attn_exact ? 1 : gqa_decode_splits(b, s, h, kvh, head_dim, cap);
    float *part = nullptr;
    uint32_t *counters = nullptr;
    if (nsplit > 1 && (int64_t)b * kvh <= B2M_ATTN_COUNTERS) {
      if (!ctx->attn_counters) {
        // Made once, outside any stream capture (a call under capture without
        // them keeps the separate merge launch).
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        B2M_CUDA(cudaStreamIsCapturing(ctx->stream, &cs));
        if (cs == cudaStreamCaptureStatusNone) {
          B2M_CUDA(cudaMalloc(&ctx->attn_counters, B2M_ATTN_COUNTERS * sizeof(uint32_t)));
          B2M_CUDA(cudaMemsetAsync(ctx->attn_counters, 0, B2M_ATTN_COUNTERS * sizeof(uint32_t), ctx->stream));
        }
      }
      counters = ctx->attn_counters;
    }
    // Without `out` (only the f16 copy wanted), kernels that form the f16
    // output themselves skip the fp32 rows; the others write them to scratch.
    const size_t out_bytes = (size_t)b * s * h * head_dim * 4;
    const bool out_scratch =
        !out && !gqa_writes_f16(q, q_rs, k_cache, v_cache, past, cos_cache, rotary_dim, b, s, h, kvh, head_dim, cap,
                                nsplit, ctx->attn_exact, counters != nullptr);
    const size_t part_bytes = nsplit > 1 ? (size_t)b * h * nsplit * (2 + head_dim) * 4 : 0;
    Scratch scr(ctx, (part_bytes || out_scratch) ? part_bytes + (out_scratch ? out_bytes : 0) + 512 : 0);
    if (nsplit > 1) part = static_cast<float *>(scr.take(part_bytes));
    if (out_scratch) out = static_cast<float *>(scr.take(out_bytes));
    launch_gqa(q, k, v, q_rs, kv_rs, k_cache, v_cache, past, cos_cache, sin_cache, rotary_half, rotary_dim,
               interleaved ? 1 : 0, out, b, s, h, kvh, head_dim, cap, sc, ctx->dev_err, part, nsplit,
               ctx->attn_exact, counters, ctx->stream, reinterpret_cast<__half *>(out16), qk_gain, qk_eps);
  });
}

B2M_API b2m_status b2m_gqa_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                               int64_t kv_rs, float *k_cache, float *v_cache, const int32_t *past,
                               const float *cos_cache, const float *sin_cache, int32_t rotary_half,
                               int32_t rotary_dim, int32_t interleaved, float *out, int32_t b, int32_t s, int32_t h,
                               int32_t kvh, int32_t head_dim, int32_t cap, float scale) {
  return gqa_impl(ctx, q, k, v, q_rs, kv_rs, k_cache, v_cache, past, cos_cache, sin_cache, rotary_half, rotary_dim,
                  interleaved, out, b, s, h, kvh, head_dim, cap, scale, nullptr);
}

B2M_API b2m_status b2m_gqa_f16_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                                   int64_t kv_rs, float *k_cache, float *v_cache, const int32_t *past,
                                   const float *cos_cache, const float *sin_cache, int32_t rotary_half,
                                   int32_t rotary_dim, int32_t interleaved, float *out, uint16_t *out16, int32_t b,
                                   int32_t s, int32_t h, int32_t kvh, int32_t head_dim, int32_t cap, float scale) {
  if (!out16) {
    b2m_set_last_error("GroupQueryAttention f16: out16 is null");
    return B2M_ERR_INVALID_ARGUMENT;
  }
  return gqa_impl(ctx, q, k, v, q_rs, kv_rs, k_cache, v_cache, past, cos_cache, sin_cache, rotary_half, rotary_dim,
                  interleaved, out, b, s, h, kvh, head_dim, cap, scale, out16);
}

B2M_API b2m_status b2m_gqa_qknorm_dev(b2m_ctx *ctx, float *q, float *k, const float *v, int64_t q_rs, int64_t kv_rs,
                                      const float *qk_gain, double eps, float *k_cache, float *v_cache,
                                      const int32_t *past, const float *cos_cache, const float *sin_cache,
                                      int32_t rotary_half, int32_t rotary_dim, int32_t interleaved, float *out,
                                      uint16_t *out16, int32_t b, int32_t s, int32_t h, int32_t kvh, int32_t head_dim,
                                      int32_t cap, float scale) {
  if ((int64_t)b * s > 0 && !qk_gain) {
    b2m_set_last_error("GroupQueryAttention q/k norm: qk_gain is null");
    return B2M_ERR_INVALID_ARGUMENT;
  }
  if (!(eps >= 0.0)) {
    b2m_set_last_error("GroupQueryAttention q/k norm: eps must be >= 0");
    return B2M_ERR_INVALID_ARGUMENT;
  }
  return gqa_impl(ctx, q, k, v, q_rs, kv_rs, k_cache, v_cache, past, cos_cache, sin_cache, rotary_half, rotary_dim,
                  interleaved, out, b, s, h, kvh, head_dim, cap, scale, out16, qk_gain, eps);
}

static b2m_status mha_impl(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                               int64_t kv_rs, const float *mask, int64_t mask_bs, int64_t mask_hs, int64_t mask_qs,
                               float *out, int32_t b, int32_t s, int32_t t, int32_t h, int32_t kvh, int32_t head_dim,
                               float scale, int32_t causal, uint16_t *planes) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(b >= 0 && s >= 0 && t > 0 && h > 0 && kvh > 0 && h % kvh == 0 && head_dim > 0 && head_dim <= 256,
                B2M_ERR_INVALID_ARGUMENT, "MultiHeadAttention: bad shape arguments");
    B2M_REQUIRE(q_rs >= (int64_t)h * head_dim && kv_rs >= (int64_t)kvh * head_dim, B2M_ERR_INVALID_ARGUMENT,
                "MultiHeadAttention: row strides too small");
    B2M_REQUIRE(mask_bs >= 0 && mask_hs >= 0 && mask_qs >= 0, B2M_ERR_INVALID_ARGUMENT,
                "MultiHeadAttention: negative mask strides");
    B2M_REQUIRE(!causal || s <= t, B2M_ERR_INVALID_ARGUMENT, "MultiHeadAttention: causal needs s <= t");
    B2M_REQUIRE((int64_t)b * s == 0 || (q && k && v && out), B2M_ERR_INVALID_ARGUMENT,
                "MultiHeadAttention: null pointer");
    B2M_REQUIRE(!planes || ((int64_t)h * head_dim) % 64 == 0, B2M_ERR_INVALID_ARGUMENT,
                "MultiHeadAttention split: h * head_dim must be a multiple of 64");
    DeviceGuard dg(ctx->device);
    if ((int64_t)b * s == 0) return;
    const float sc = scale > 0.f ? scale : 1.f / std::sqrt((float)head_dim);
    launch_mha(q, k, v, q_rs, kv_rs, mask, mask_bs, mask_hs, mask_qs, out, b, s, t, h, kvh, head_dim, sc,
               causal ? 1 : 0, ctx->dev_err, ctx->attn_exact, ctx->stream, reinterpret_cast<__nv_bfloat16 *>(planes));
  });
}

B2M_API b2m_status b2m_mha_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                               int64_t kv_rs, const float *mask, int64_t mask_bs, int64_t mask_hs, int64_t mask_qs,
                               float *out, int32_t b, int32_t s, int32_t t, int32_t h, int32_t kvh, int32_t head_dim,
                               float scale, int32_t causal) {
  return mha_impl(ctx, q, k, v, q_rs, kv_rs, mask, mask_bs, mask_hs, mask_qs, out, b, s, t, h, kvh, head_dim, scale,
                  causal, nullptr);
}

B2M_API b2m_status b2m_mha_split_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                                     int64_t kv_rs, const float *mask, int64_t mask_bs, int64_t mask_hs,
                                     int64_t mask_qs, float *out, uint16_t *out_planes, int32_t b, int32_t s,
                                     int32_t t, int32_t h, int32_t kvh, int32_t head_dim, float scale,
                                     int32_t causal) {
  if (!out_planes) {
    b2m_set_last_error("MultiHeadAttention split: out_planes is null");
    return B2M_ERR_INVALID_ARGUMENT;
  }
  return mha_impl(ctx, q, k, v, q_rs, kv_rs, mask, mask_bs, mask_hs, mask_qs, out, b, s, t, h, kvh, head_dim, scale,
                  causal, out_planes);
}

B2M_API b2m_status b2m_dynamic_quantize_linear_dev(b2m_ctx *ctx, const float *x, int64_t n, uint8_t *y,
                                                   float *scale, uint8_t *zero_point) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(n >= 0 && scale && zero_point && (n == 0 || (x && y)), B2M_ERR_INVALID_ARGUMENT,
                "DynamicQuantizeLinear: bad arguments");
    DeviceGuard dg(ctx->device);
    const size_t need = dql_partial_floats() * sizeof(float);
    Scratch sc(ctx, need + 256);
    launch_dynamic_quantize(x, n, y, scale, zero_point, static_cast<float *>(sc.take(need)), ctx->dev_counter,
                            ctx->stream);
  });
}

B2M_API b2m_status b2m_rotary_dev(b2m_ctx *ctx, const float *x, int64_t x_rs, const int64_t *positions,
                                  int32_t pos_per_batch, const float *cos_cache, const float *sin_cache,
                                  int32_t half, int32_t max_pos, float *y, int64_t y_rs, int32_t b, int32_t s,
                                  int32_t heads, int32_t head_dim, int32_t rotary_dim, int32_t interleaved) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(b >= 0 && s >= 0 && heads > 0 && head_dim > 0 && head_dim <= 256 && half > 0 && max_pos > 0,
                B2M_ERR_INVALID_ARGUMENT, "RotaryEmbedding: bad shape arguments");
    B2M_REQUIRE(rotary_dim > 0 && rotary_dim % 2 == 0 && rotary_dim <= head_dim && rotary_dim / 2 <= half,
                B2M_ERR_INVALID_ARGUMENT, "RotaryEmbedding: bad rotary_dim");
    B2M_REQUIRE(x_rs >= (int64_t)heads * head_dim && y_rs >= (int64_t)heads * head_dim, B2M_ERR_INVALID_ARGUMENT,
                "RotaryEmbedding: row strides too small");
    B2M_REQUIRE((int64_t)b * s == 0 || (x && y && positions && cos_cache && sin_cache), B2M_ERR_INVALID_ARGUMENT,
                "RotaryEmbedding: null pointer");
    DeviceGuard dg(ctx->device);
    launch_rotary(x, x_rs, positions, pos_per_batch ? 1 : 0, cos_cache, sin_cache, half, max_pos, y, y_rs, b, s,
                  heads, head_dim, rotary_dim, interleaved ? 1 : 0, ctx->dev_err, ctx->stream);
  });
}

B2M_API b2m_status b2m_advance_positions_dev(b2m_ctx *ctx, int32_t *past, int32_t n, int32_t delta) {
  return guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(n >= 0 && (n == 0 || past), B2M_ERR_INVALID_ARGUMENT, "advance positions: bad arguments");
    DeviceGuard dg(ctx->device);
    launch_advance_positions(past, n, delta, ctx->stream);
  });
}

// ---------------------------------------------------------------------------
// Conv / ConvInteger / QLinearConv: im2col panels on the device feeding the
// fp32 and int8 GEMM kernels (opConv, lib/src/onnx_nn_ops.dart:179-545;
// opConvInteger / opQLinearConv, lib/src/onnx_qlinear_ops.dart:230-382).
// ---------------------------------------------------------------------------

namespace {

// Bytes of im2col panel (or GEMM output) one pass may hold; images beyond it
// run in further passes over the same scratch.
constexpr int64_t CONV_PANEL_BYTES = (int64_t)512 << 20;

// Spatial attributes of one call, resolved as _resolvePads
// (onnx_nn_ops.dart:38-88, no ceil mode) into a ConvGeom.
ConvGeom conv_geometry(const b2m_tensor *x, int64_t m, int64_t wk, const int64_t *kernel_shape,
                       const int64_t *strides, const int64_t *pads, const int64_t *dilations, int32_t group,
                       int32_t auto_pad, const char *op) {
  const int nd = x->rank - 2;
  B2M_REQUIRE(kernel_shape, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": kernel_shape is required");
  B2M_REQUIRE(group >= 1, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": group must be >= 1");
  B2M_REQUIRE(auto_pad >= B2M_AUTO_PAD_NOTSET && auto_pad <= B2M_AUTO_PAD_VALID, B2M_ERR_INVALID_ARGUMENT,
              std::string(op) + ": bad auto_pad");
  ConvGeom g;
  g.n = x->shape[0];
  g.cin = x->shape[1];
  g.m = m;
  g.group = group;
  int64_t kvol = 1;
  for (int a = 0; a < nd; a++) {
    B2M_REQUIRE(kernel_shape[a] >= 1, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": bad kernel_shape");
    kvol *= kernel_shape[a];
  }
  B2M_REQUIRE(wk % kvol == 0, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": weight does not match kernel_shape");
  g.cpg = wk / kvol;
  B2M_REQUIRE(g.cin == g.cpg * group, B2M_ERR_INVALID_ARGUMENT,
              std::string(op) + " channel mismatch: input C=" + std::to_string(g.cin) +
                  ", weight C/g=" + std::to_string(g.cpg) + ", group=" + std::to_string(group));
  B2M_REQUIRE(m % group == 0, B2M_ERR_INVALID_ARGUMENT,
              std::string(op) + ": output channels " + std::to_string(m) + " not divisible by group");
  g.mpg = m / group;
  g.K = wk;
  g.P = 1;
  const int off = 3 - nd;  // spatial axis a of the call is axis off + a of the geometry
  for (int a = 0; a < nd; a++) {
    const int64_t in = x->shape[2 + a], k = kernel_shape[a];
    const int64_t s = strides ? strides[a] : 1, d = dilations ? dilations[a] : 1;
    B2M_REQUIRE(s >= 1 && d >= 1, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": strides / dilations must be >= 1");
    const int64_t window = d * (k - 1) + 1;
    int64_t pb = 0, out = 0;
    if (auto_pad == B2M_AUTO_PAD_SAME_UPPER || auto_pad == B2M_AUTO_PAD_SAME_LOWER) {
      out = (in + s - 1) / s;
      const int64_t total = std::max<int64_t>(0, (out - 1) * s + window - in);
      const int64_t small = total / 2;
      pb = auto_pad == B2M_AUTO_PAD_SAME_UPPER ? small : total - small;
    } else if (auto_pad == B2M_AUTO_PAD_VALID) {
      out = in >= window ? (in - window) / s + 1 : 0;
    } else {
      pb = pads ? pads[a] : 0;
      const int64_t pe = pads ? pads[nd + a] : 0;
      B2M_REQUIRE(pb >= 0 && pe >= 0, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": pads must be >= 0");
      const int64_t span = in + pb + pe - window;
      out = span >= 0 ? span / s + 1 : 0;
    }
    B2M_REQUIRE(out >= 1, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": empty output along a spatial axis");
    g.in[off + a] = in;
    g.k[off + a] = k;
    g.st[off + a] = s;
    g.dil[off + a] = d;
    g.pad[off + a] = pb;
    g.out[off + a] = out;
    g.P *= out;
  }
  const int64_t lim = INT32_MAX;
  B2M_REQUIRE(g.K < lim && g.P < lim && g.cin < lim && g.m < lim && g.cpg * g.in[0] * g.in[1] * g.in[2] < lim,
              B2M_ERR_UNSUPPORTED, std::string(op) + ": dimensions beyond 2^31 (per image and group)");
  return g;
}

std::vector<int64_t> conv_out_shape(const ConvGeom &g, int nd) {
  std::vector<int64_t> s = {g.n, g.m};
  for (int a = 3 - nd; a < 3; a++) s.push_back(g.out[a]);
  return s;
}

// Images per pass so that `bytes_per_image` x images stays within the panel
// budget (at least one).
int64_t images_per_pass(const ConvGeom &g, int64_t bytes_per_image, int64_t max_rows_per_image = 0) {
  int64_t nb = std::max<int64_t>(1, CONV_PANEL_BYTES / std::max<int64_t>(1, bytes_per_image));
  if (max_rows_per_image > 0) nb = std::min<int64_t>(nb, std::max<int64_t>(1, ((int64_t)1 << 21) / max_rows_per_image));
  return std::min<int64_t>(nb, g.n);
}

void conv_f32_impl(b2m_ctx *ctx, const b2m_tensor *x, const b2m_weight *w, const b2m_tensor *bias,
                   const int64_t *kernel_shape, const int64_t *strides, const int64_t *pads, const int64_t *dilations,
                   int32_t group, int32_t auto_pad, int32_t mode, b2m_tensor **y) {
  require_float(x, "Conv input");
  B2M_REQUIRE(x->rank >= 3 && x->rank <= 5, B2M_ERR_UNSUPPORTED,
              "Conv supports 1-3 spatial dims, got rank " + std::to_string(x->rank));
  B2M_REQUIRE(w && w->kind == W_F32, B2M_ERR_INVALID_ARGUMENT, "Conv: w is not an fp32 conv weight");
  B2M_REQUIRE(mode == B2M_MODE_EXACT || mode == B2M_MODE_FAST, B2M_ERR_INVALID_ARGUMENT, "Conv: bad mode");
  const int nd = x->rank - 2;
  const ConvGeom g = conv_geometry(x, w->n, w->k, kernel_shape, strides, pads, dilations, group, auto_pad, "Conv");
  if (bias) {
    require_float(bias, "Conv bias");
    B2M_REQUIRE(bias->numel == g.m, B2M_ERR_INVALID_ARGUMENT, "Conv: bias must have one value per output channel");
  }
  check_cancel(ctx);
  b2m_tensor *out = prepare_output(ctx, y, B2M_FLOAT, conv_out_shape(g, nd));
  if (out->numel == 0) return;
  OpTimer timer(ctx);
  const float *xd = static_cast<const float *>(x->data);
  const float *bd = bias ? static_cast<const float *>(bias->data) : nullptr;
  float *yd = static_cast<float *>(out->data);
  // The reference's direct double paths: depthwise 1-D / 2-D (padded taps
  // included, onnx_nn_ops.dart:423-483) and every 3-D conv (:485-530).
  const bool depthwise = nd <= 2 && g.cpg == 1 && g.mpg == 1;
  if (nd == 3 || depthwise) {
    launch_conv_direct_double(xd, w->f32, bd, g, depthwise ? 1 : 0, yd, ctx->stream);
    timer.done();
    return;
  }
  const int64_t plane = g.in[0] * g.in[1] * g.in[2];
  if (mode == B2M_MODE_FAST && w->bx_hi) {
    const int64_t kp = f32_tc_kp(g.K);
    const int64_t nb = images_per_pass(g, g.P * kp * 4, g.P);
    Scratch sc(ctx, (size_t)(nb * g.P * kp * 4) + 512);
    void *planes = sc.take((size_t)(nb * g.P * kp * 4));
    const uint16_t *hi_planes = w->bx_hi, *lo_planes = w->bx_lo;
    for (int64_t b0 = 0; b0 < g.n; b0 += nb) {
      const int64_t cnt = std::min(nb, g.n - b0);
      for (int64_t grp = 0; grp < g.group; grp++) {
        void *hi = planes;
        void *lo = static_cast<uint16_t *>(planes) + cnt * g.P * kp;
        launch_conv_im2col_planes(xd, g, grp, b0, cnt, kp, hi, lo, ctx->stream);
        F32GemmArgs p;
        p.M = cnt * g.P;
        p.N = g.mpg;
        p.K = g.K;
        p.Y = yd + (b0 * g.m + grp * g.mpg) * g.P;
        p.ldy = g.P;
        p.epi = EPI_GEMM;
        if (bd) {
          p.C = bd + grp * g.mpg;
          p.c_rs = 0;
          p.c_cs = 1;
        }
        p.dev_err = ctx->dev_err;
        launch_f32_tc_planes(p, hi_planes + grp * g.mpg * kp, lo_planes + grp * g.mpg * kp, g.mpg, planes, g.P,
                             g.m * g.P, ctx->stream);
      }
    }
    timer.done();
    return;
  }
  // EXACT: Y_g[mpg][P] = W_g[mpg][K] . panel[K][P] per image, the reference's
  // matmulKernel(W_g, cols) with the chunk of output rows as the call's
  // columns (chunkRows = (8 << 20) floats / (K * ow), onnx_nn_ops.dart:313-323),
  // then the bias in float32 (:406-418).
  const int64_t ow = g.out[2], oh = g.out[1] * g.out[0];
  const int64_t chunk_rows = std::min<int64_t>(oh, std::max<int64_t>(1, ((int64_t)8 << 20) / (g.K * ow)));
  const bool pointwise = nd <= 2 && g.K == g.cpg && g.st[1] == 1 && g.st[2] == 1 && g.pad[1] == 0 &&
                         g.pad[2] == 0 && g.out[1] == g.in[1] && g.out[2] == g.in[2];
  const int64_t nb = pointwise ? g.n : std::min<int64_t>(images_per_pass(g, g.K * g.P * 4), 65535);
  Scratch sc(ctx, pointwise ? 0 : (size_t)(nb * g.K * g.P * 4) + 256);
  float *cols = pointwise ? nullptr : static_cast<float *>(sc.take((size_t)(nb * g.K * g.P * 4)));
  for (int64_t b0 = 0; b0 < g.n; b0 += nb) {
    const int64_t cnt = std::min(nb, g.n - b0);
    for (int64_t grp = 0; grp < g.group; grp++) {
      F32GemmArgs p;
      p.A = w->f32 + grp * g.mpg;  // W_g(i, k) = W^T[k][grp * mpg + i]
      p.sa_m = 1;
      p.sa_k = g.m;
      if (pointwise) {
        p.B = xd + (b0 * g.cin + grp * g.cpg) * plane;
        p.b_bstride[0] = g.cin * plane;
      } else {
        launch_conv_im2col_f32(xd, g, grp, b0, cnt, cols, ctx->stream);
        p.B = cols;
        p.b_bstride[0] = g.K * g.P;
      }
      p.sb_k = g.P;
      p.sb_n = 1;
      p.Y = yd + (b0 * g.m + grp * g.mpg) * g.P;
      p.ldy = g.P;
      p.M = g.mpg;
      p.N = g.P;
      p.K = g.K;
      p.nbd = 1;
      p.bdims[0] = cnt;
      p.a_bstride[0] = 0;
      p.y_bstride = g.m * g.P;
      p.batch = cnt;
      p.m_eff = g.mpg;
      p.tile_w = chunk_rows * ow;
      p.epi = EPI_GEMM;
      if (bd) {
        p.C = bd + grp * g.mpg;
        p.c_rs = 1;
        p.c_cs = 0;
      }
      p.dev_err = ctx->dev_err;
      launch_f32_exact(p, ctx->stream);
    }
  }
  timer.done();
}

void conv_int_impl(b2m_ctx *ctx, const b2m_tensor *x, const b2m_tensor *xzp, const b2m_weight *w,
                   const b2m_tensor *wzp, const int64_t *kernel_shape, const int64_t *strides, const int64_t *pads,
                   const int64_t *dilations, int32_t group, bool requant, double xs, const b2m_tensor *ws,
                   double ys, int32_t yzp, const b2m_tensor *bias, int32_t lo, int32_t hi, b2m_tensor **y) {
  const char *op = requant ? "QLinearConv" : "ConvInteger";
  B2M_REQUIRE(x && is_i8(x->dtype), B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": x must be uint8 or int8");
  if (requant)
    B2M_REQUIRE(x->rank == 4, B2M_ERR_UNSUPPORTED, "QLinearConv implemented for 2-D convs");
  else
    B2M_REQUIRE(x->rank == 3 || x->rank == 4, B2M_ERR_UNSUPPORTED, "ConvInteger implemented for 1-D/2-D convs");
  B2M_REQUIRE(w && w->kind == W_I8, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": w is not an int8 conv weight");
  const int nd = x->rank - 2;
  int64_t kvol = 1;
  B2M_REQUIRE(kernel_shape, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": kernel_shape is required");
  for (int a = 0; a < nd; a++) kvol *= std::max<int64_t>(1, kernel_shape[a]);
  B2M_REQUIRE(group >= 1 && x->shape[1] % group == 0, B2M_ERR_INVALID_ARGUMENT,
              std::string(op) + ": input channels not divisible by group");
  const int64_t K = x->shape[1] / group * kvol;
  B2M_REQUIRE(w->k == K || w->k == round_up(K, 16), B2M_ERR_INVALID_ARGUMENT,
              std::string(op) + ": weight does not match the input channels and kernel_shape");
  const ConvGeom g = conv_geometry(x, w->n, K, kernel_shape, strides, pads, dilations, group, B2M_AUTO_PAD_NOTSET, op);
  if (wzp && wzp->numel != 1 && wzp->numel != g.m)
    b2m_throw(B2M_ERR_UNSUPPORTED, "ConvInteger: weight zero point must be scalar or per-output-channel");
  if (wzp) B2M_REQUIRE(wzp->dtype == w->i8.dtype, B2M_ERR_INVALID_ARGUMENT, std::string(op) + ": w_zero_point dtype");
  if (xzp) B2M_REQUIRE(xzp->dtype == x->dtype && xzp->numel >= 1, B2M_ERR_INVALID_ARGUMENT,
                       std::string(op) + ": x_zero_point dtype");
  B2M_REQUIRE(w->k <= 33025, B2M_ERR_UNSUPPORTED, std::string(op) + ": a reduction beyond 33025 may leave int32");
  int32_t odt = B2M_INT32;
  if (requant) {
    B2M_REQUIRE((lo == 0 && hi == 255) || (lo == -128 && hi == 127), B2M_ERR_INVALID_ARGUMENT,
                "QLinearConv: lo/hi must be [0,255] or [-128,127]");
    B2M_REQUIRE(ws && ws->dtype == B2M_FLOAT && (ws->numel == 1 || ws->numel == g.m), B2M_ERR_INVALID_ARGUMENT,
                "QLinearConv: w_scale must be float with 1 or M values");
    if (bias)
      B2M_REQUIRE(bias->dtype == B2M_INT32 && bias->numel == g.m, B2M_ERR_INVALID_ARGUMENT,
                  "QLinearConv: bias must be int32 with one value per output channel");
    odt = lo == 0 ? B2M_UINT8 : B2M_INT8;
  }
  check_cancel(ctx);
  b2m_tensor *out = prepare_output(ctx, y, odt, conv_out_shape(g, nd));
  if (out->numel == 0) return;
  OpTimer timer(ctx);
  const int64_t kg = w->k;
  const int64_t nb = images_per_pass(g, g.P * (kg + 4 * g.mpg + 4), g.P);
  const size_t rows_b = (size_t)(nb * g.P * kg), z_b = (size_t)(nb * g.P * g.mpg * 4), rs_b = (size_t)(nb * g.P * 4);
  Scratch sc(ctx, rows_b + z_b + rs_b + 3 * 256);
  uint8_t *rows = static_cast<uint8_t *>(sc.take(rows_b));
  int32_t *z = static_cast<int32_t *>(sc.take(z_b));
  int32_t *rowsum = static_cast<int32_t *>(sc.take(rs_b));
  ConvRequant rq;
  if (requant) {
    rq.xs = xs;
    rq.ys = ys;
    rq.ws = static_cast<const float *>(ws->data);
    rq.ws_len = ws->numel;
    rq.bias = bias ? static_cast<const int32_t *>(bias->data) : nullptr;
    rq.y_zp = yzp;
    rq.lo = lo;
    rq.hi = hi;
  }
  const bool per_channel = wzp && wzp->numel == g.m && g.m != 1;
  for (int64_t b0 = 0; b0 < g.n; b0 += nb) {
    const int64_t cnt = std::min(nb, g.n - b0);
    for (int64_t grp = 0; grp < g.group; grp++) {
      launch_conv_im2col_i8(x->data, g, grp, b0, cnt, kg, xzp ? xzp->data : nullptr, rows, ctx->stream);
      I8GemmArgs p;
      p.A = rows;
      p.a_signed = x->dtype == B2M_INT8;
      p.Bt = w->i8.bt + grp * g.mpg * w->i8.kpad;
      p.b_signed = w->i8.dtype == B2M_INT8;
      p.kpad = w->i8.kpad;
      p.colsum = w->i8.colsum + grp * g.mpg;
      if (xzp) {
        p.azp = xzp->data;
        p.azp_len = 1;
        p.azp_signed = xzp->dtype == B2M_INT8;
      }
      if (wzp) {
        p.bzp = static_cast<const uint8_t *>(wzp->data) + (per_channel ? grp * g.mpg : 0);
        p.bzp_len = per_channel ? g.mpg : 1;
        p.bzp_signed = wzp->dtype == B2M_INT8;
      }
      p.M = cnt * g.P;
      p.N = g.mpg;
      p.K = kg;
      p.batch = 1;
      p.Y32 = z;
      p.rowsum = rowsum;
      p.dev_err = ctx->dev_err;
      const bool done = g.group == 1 && launch_i8_tc(p, w->i8, ctx->stream);
      if (!done) launch_i8_gemm(p, ctx->stream);
      launch_conv_scatter(z, g, grp, b0, cnt, requant ? nullptr : static_cast<int32_t *>(out->data),
                          requant ? out->data : nullptr, rq, ctx->stream);
    }
  }
  timer.done();
}

// ConvTranspose (opConvTranspose, onnx_nn_ops.dart:815-1060): the
// reference's two arithmetics, in EXACT terms for every call.
void conv_transpose_impl(b2m_ctx *ctx, const b2m_tensor *x, const b2m_tensor *w, const b2m_tensor *bias,
                         const int64_t *strides, const int64_t *pads, const int64_t *dilations,
                         const int64_t *output_padding, const int64_t *output_shape, int32_t group, b2m_tensor **y) {
  require_float(x, "ConvTranspose input");
  require_float(w, "ConvTranspose weight");
  B2M_REQUIRE(x->rank >= 3 && x->rank <= 5, B2M_ERR_UNSUPPORTED,
              "ConvTranspose supports 1-3 spatial dims, got rank " + std::to_string(x->rank));
  B2M_REQUIRE(w->rank == x->rank, B2M_ERR_INVALID_ARGUMENT, "ConvTranspose weight rank must match input rank");
  const int nd = x->rank - 2;
  B2M_REQUIRE(group >= 1 && x->shape[1] % group == 0 && w->shape[0] == x->shape[1], B2M_ERR_INVALID_ARGUMENT,
              "ConvTranspose channel mismatch: input C=" + std::to_string(x->shape[1]) + ", weight C=" +
                  std::to_string(w->shape[0]) + ", group=" + std::to_string(group));
  ConvTGeom g;
  g.n = x->shape[0];
  g.cin = x->shape[1];
  g.group = group;
  g.cpg = g.cin / group;
  g.mpg = w->shape[1];
  g.m = g.mpg * group;
  const int off = 3 - nd;
  for (int a = 0; a < nd; a++) {
    const int64_t in = x->shape[2 + a], k = w->shape[2 + a];
    const int64_t s = strides ? strides[a] : 1, d = dilations ? dilations[a] : 1;
    const int64_t op = output_padding ? output_padding[a] : 0;
    B2M_REQUIRE(s >= 1 && d >= 1 && op >= 0 && k >= 1, B2M_ERR_INVALID_ARGUMENT,
                "ConvTranspose: strides / dilations must be >= 1, output_padding >= 0");
    const int64_t full = (in - 1) * s + d * (k - 1) + 1 + op;
    int64_t pb = pads ? pads[a] : 0, pe = pads ? pads[nd + a] : 0, out;
    if (output_shape) {
      // The spec's split of the difference, the larger half at the start.
      out = output_shape[a];
      const int64_t total = full - out;
      pe = total / 2;
      pb = total - pe;
    } else {
      B2M_REQUIRE(pb >= 0 && pe >= 0, B2M_ERR_INVALID_ARGUMENT, "ConvTranspose: pads must be >= 0");
      out = full - pb - pe;
    }
    B2M_REQUIRE(out >= 1, B2M_ERR_INVALID_ARGUMENT, "ConvTranspose: empty output along a spatial axis");
    g.in[off + a] = in;
    g.k[off + a] = k;
    g.st[off + a] = s;
    g.dil[off + a] = d;
    g.pad[off + a] = pb;
    g.out[off + a] = out;
  }
  if (bias) {
    require_float(bias, "ConvTranspose bias");
    B2M_REQUIRE(bias->numel == g.m, B2M_ERR_INVALID_ARGUMENT,
                "ConvTranspose: bias must have one value per output channel");
  }
  check_cancel(ctx);
  std::vector<int64_t> oshape = {g.n, g.m};
  for (int a = off; a < 3; a++) oshape.push_back(g.out[a]);
  b2m_tensor *out = prepare_output(ctx, y, B2M_FLOAT, oshape);
  if (out->numel == 0) return;
  OpTimer timer(ctx);
  const float *xd = static_cast<const float *>(x->data), *wd = static_cast<const float *>(w->data);
  const float *bd = bias ? static_cast<const float *>(bias->data) : nullptr;
  float *yd = static_cast<float *>(out->data);
  if (nd <= 2 && !output_shape && g.n == 1) {
    // GEMM path (:850-963): prod[mpg*kvol][H*W] = W_g^T . X_g, then overlap-add.
    const int64_t kvol = g.k[1] * g.k[2], mk = g.mpg * kvol, hw = g.in[1] * g.in[2];
    B2M_REQUIRE(mk <= 65535, B2M_ERR_UNSUPPORTED, "ConvTranspose: too many output planes per group");
    Scratch sc(ctx, (size_t)(mk * hw * 4) + 256);
    float *prod = static_cast<float *>(sc.take((size_t)(mk * hw * 4)));
    for (int64_t grp = 0; grp < g.group; grp++) {
      F32GemmArgs p;
      p.A = wd + grp * g.cpg * mk;  // A(i, c) = W[grp * cpg + c][i]
      p.sa_m = 1;
      p.sa_k = mk;
      p.B = xd + grp * g.cpg * hw;
      p.sb_k = hw;
      p.sb_n = 1;
      p.Y = prod;
      p.ldy = hw;
      p.M = mk;
      p.N = hw;
      p.K = g.cpg;
      p.batch = 1;
      p.m_eff = mk;
      p.tile_w = hw;
      p.epi = EPI_NONE;
      p.dev_err = ctx->dev_err;
      launch_f32_exact(p, ctx->stream);
      launch_conv_transpose_col2im(prod, g, grp, bd, yd, ctx->stream);
    }
  } else {
    launch_conv_transpose_scatter(xd, wd, bd, g, yd, ctx->stream);
  }
  timer.done();
}

}  // namespace

extern "C" {

B2M_API b2m_status b2m_conv_transpose_f32(b2m_ctx *ctx, const b2m_tensor *x, const b2m_tensor *w,
                                          const b2m_tensor *bias, const int64_t *strides, const int64_t *pads,
                                          const int64_t *dilations, const int64_t *output_padding,
                                          const int64_t *output_shape, int32_t group, b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    conv_transpose_impl(ctx, x, w, bias, strides, pads, dilations, output_padding, output_shape, group, y);
  });
}

B2M_API b2m_status b2m_weight_prepack_conv(b2m_ctx *ctx, const void *host_w, int32_t dtype, int64_t m, int64_t k,
                                           b2m_weight **out) {
  if (dtype == B2M_FLOAT) return b2m_weight_prepack_f32(ctx, static_cast<const float *>(host_w), m, k, 1, out);
  b2m_status st = guarded([&] {
    check_ctx(ctx);
    B2M_REQUIRE(out && host_w && m > 0 && k > 0, B2M_ERR_INVALID_ARGUMENT, "Conv prepack: bad arguments");
    B2M_REQUIRE(is_i8(dtype), B2M_ERR_INVALID_ARGUMENT, "Conv prepack: dtype must be float, uint8 or int8");
  });
  if (st != B2M_OK) return st;
  // W [m][k] -> W^T [kg][m], k zero-padded to a multiple of 16.
  const int64_t kg = (k + 15) / 16 * 16;
  std::vector<uint8_t> bt;
  st = guarded([&] {
    bt.assign((size_t)(kg * m), 0);
    const uint8_t *src = static_cast<const uint8_t *>(host_w);
    for (int64_t j = 0; j < m; j++)
      for (int64_t kk = 0; kk < k; kk++) bt[(size_t)(kk * m + j)] = src[j * k + kk];
  });
  if (st != B2M_OK) return st;
  return b2m_weight_prepack_i8(ctx, bt.data(), dtype, kg, m, out);
}

B2M_API b2m_status b2m_conv_f32(b2m_ctx *ctx, const b2m_tensor *x, const b2m_weight *w, const b2m_tensor *bias,
                                const int64_t *kernel_shape, const int64_t *strides, const int64_t *pads,
                                const int64_t *dilations, int32_t group, int32_t auto_pad, int32_t mode,
                                b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    conv_f32_impl(ctx, x, w, bias, kernel_shape, strides, pads, dilations, group, auto_pad, mode, y);
  });
}

B2M_API b2m_status b2m_conv_integer(b2m_ctx *ctx, const b2m_tensor *x, const b2m_tensor *x_zp, const b2m_weight *w,
                                    const b2m_tensor *w_zp, const int64_t *kernel_shape, const int64_t *strides,
                                    const int64_t *pads, const int64_t *dilations, int32_t group, b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    conv_int_impl(ctx, x, x_zp, w, w_zp, kernel_shape, strides, pads, dilations, group, false, 0.0, nullptr, 1.0, 0,
                  nullptr, 0, 0, y);
  });
}

B2M_API b2m_status b2m_qlinear_conv(b2m_ctx *ctx, const b2m_tensor *x, float x_scale, const b2m_tensor *x_zp,
                                    const b2m_weight *w, const b2m_tensor *w_scale,
                                    const b2m_tensor *w_zp, float y_scale, int32_t y_zp, const b2m_tensor *bias,
                                    const int64_t *kernel_shape, const int64_t *strides, const int64_t *pads,
                                    const int64_t *dilations, int32_t group, int32_t lo, int32_t hi, b2m_tensor **y) {
  return guarded([&] {
    check_ctx(ctx);
    DeviceGuard dg(ctx->device);
    conv_int_impl(ctx, x, x_zp, w, w_zp, kernel_shape, strides, pads, dilations, group, true, (double)x_scale,
                  w_scale, (double)y_scale, y_zp, bias, lo, hi, y);
  });
}

}  // extern "C"
