// Convolution kernels: the im2col panels that turn Conv / ConvInteger /
// QLinearConv into GEMMs on the existing cores, the direct double-accumulated
// convolution of the reference's depthwise and N-D paths, and the scatter of
// integer GEMM results into NC[D]HW with QLinearConv's requantisation.
//
// Reference: opConv (lib/src/onnx_nn_ops.dart:179-545), _convIntAcc /
// opConvInteger / opQLinearConv (lib/src/onnx_qlinear_ops.dart:230-382).
//
// Index decomposition: GEMM reduction index k = ((c * kD + kz) * kH + ky) * kW
// + kx, the order of the weight tensor [M][C/g][kD][kH][kW] and of the
// reference's im2col rows; pixel p = (oz * oH + oy) * oW + ox. Input
// coordinate along an axis: o * stride - pad + tap * dilation.
#include <cuda_bf16.h>

#include <algorithm>
#include <climits>

#include "b2m_internal.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

// 32-bit copies of the geometry for the index arithmetic of the kernels (the
// host checks that every extent fits).
struct Geo32 {
  int cin, cpg, mpg, m;
  int in0, in1, in2;
  int k0, k1, k2;
  int s0, s1, s2;
  int d0, d1, d2;
  int p0, p1, p2;
  int o1, o2;  // output H, W
  int K, P;
};

Geo32 geo32(const ConvGeom &g) {
  Geo32 r;
  r.cin = (int)g.cin, r.cpg = (int)g.cpg, r.mpg = (int)g.mpg, r.m = (int)g.m;
  r.in0 = (int)g.in[0], r.in1 = (int)g.in[1], r.in2 = (int)g.in[2];
  r.k0 = (int)g.k[0], r.k1 = (int)g.k[1], r.k2 = (int)g.k[2];
  r.s0 = (int)g.st[0], r.s1 = (int)g.st[1], r.s2 = (int)g.st[2];
  r.d0 = (int)g.dil[0], r.d1 = (int)g.dil[1], r.d2 = (int)g.dil[2];
  r.p0 = (int)g.pad[0], r.p1 = (int)g.pad[1], r.p2 = (int)g.pad[2];
  r.o1 = (int)g.out[1], r.o2 = (int)g.out[2];
  r.K = (int)g.K, r.P = (int)g.P;
  return r;
}

// Where tap k of the reduction reads, relative to a pixel's window origin:
// the linear offset inside the image's group-channel block (channel plane
// plus kernel offsets; 32-bit, the host keeps the block below 2^31 elements)
// and the kernel offsets along the three axes for the bounds test. A k past
// K gets dz = INT_MIN / 2, which fails every bounds test.
struct Tap {
  int off, dz, dy, dx;
};

__device__ __forceinline__ Tap make_tap(const Geo32 &g, int k) {
  Tap t;
  if (k >= g.K) {
    t.off = 0;
    t.dz = INT_MIN / 2;
    t.dy = t.dx = 0;
    return t;
  }
  const int kvol = g.k0 * g.k1 * g.k2;
  const int c = k / kvol, r = k - c * kvol;
  const int kz = r / (g.k1 * g.k2), ky = (r / g.k2) % g.k1, kx = r % g.k2;
  t.dz = kz * g.d0;
  t.dy = ky * g.d1;
  t.dx = kx * g.d2;
  t.off = ((c * g.in0 + t.dz) * g.in1 + t.dy) * g.in2 + t.dx;
  return t;
}

// A pixel's window origin (o * stride - pad along each axis) and its linear
// offset (may be negative; only in-bounds taps are ever added to it).
struct Win {
  int bz, by, bx, base;
};

__device__ __forceinline__ Win make_win(const Geo32 &g, int p) {
  const int oz = p / (g.o1 * g.o2), oy = (p / g.o2) % g.o1, ox = p % g.o2;
  Win w;
  w.bz = oz * g.s0 - g.p0;
  w.by = oy * g.s1 - g.p1;
  w.bx = ox * g.s2 - g.p2;
  w.base = (w.bz * g.in1 + w.by) * g.in2 + w.bx;
  return w;
}

// Offset of a tap of a pixel inside its image's group-channel block, or -1
// when the tap falls in the padding (or past K).
__device__ __forceinline__ int tap_at(const Geo32 &g, const Win &w, int off, int dz, int dy, int dx) {
  if ((unsigned)(w.bz + dz) >= (unsigned)g.in0 || (unsigned)(w.by + dy) >= (unsigned)g.in1 ||
      (unsigned)(w.bx + dx) >= (unsigned)g.in2)
    return -1;
  return w.base + off;
}

constexpr int TR = 32;  // panel rows (pixels) per tile
constexpr int TK = 64;  // reduction columns per tile

// The taps of one tile's reduction columns, in shared memory.
struct TapTable {
  int4 t[TK];  // off, dz, dy, dx
};

__device__ __forceinline__ void fill_taps(TapTable &tt, const Geo32 &g, int k0) {
  if (threadIdx.x < TK) {
    const Tap t = make_tap(g, k0 + threadIdx.x);
    tt.t[threadIdx.x] = make_int4(t.off, t.dz, t.dy, t.dx);
  }
}

__device__ __forceinline__ int tap_of(const TapTable &tt, const Geo32 &g, const Win &w, int kk) {
  const int4 t = tt.t[kk];
  return tap_at(g, w, t.x, t.y, t.z, t.w);
}

// fp32 panel [nb][K][P]: block (x: 256 pixels, y: 64 k rows, z: image). Each
// thread decomposes its pixel once and walks the block's 64 taps from a
// shared table; along a row of taps consecutive threads read and write
// consecutive pixels.
__global__ void __launch_bounds__(256) conv_im2col_f32_kernel(const float *__restrict__ x, const Geo32 g, int64_t grp,
                                                              int64_t b0, float *__restrict__ cols) {
  __shared__ TapTable tt;
  const int64_t plane = (int64_t)g.in0 * g.in1 * g.in2;
  const int k0 = blockIdx.y * TK;
  fill_taps(tt, g, k0);
  __syncthreads();
  const int p = blockIdx.x * 256 + threadIdx.x;
  if (p >= g.P) return;
  const int64_t img = blockIdx.z;
  const float *xb = x + ((b0 + img) * g.cin + grp * g.cpg) * plane;
  const Win w = make_win(g, p);
  float *dst = cols + (img * g.K + k0) * (int64_t)g.P + p;
  const int kn = min(TK, g.K - k0);
  for (int kk = 0; kk < kn; kk++, dst += g.P) {
    const int off = tap_of(tt, g, w, kk);
    *dst = off < 0 ? 0.f : __ldg(xb + off);
  }
}

// bf16 split planes [rows][kp]: a CTA owns 32 pixels (lane = pixel, so the
// gathers of a warp read consecutive pixels) and walks all of kp in tiles of
// 64 k; the pixel is decomposed once, the tile's taps come from a shared
// table. Each thread splits pairs of consecutive k into bf16x2 words, kept in
// shared memory with an odd word pitch (conflict-free), and each warp then
// writes whole 128-byte row segments of both planes.
__global__ void __launch_bounds__(256) conv_im2col_planes_kernel(const float *__restrict__ x, const Geo32 g,
                                                                 int64_t grp, int64_t b0, int rows, int kp,
                                                                 __nv_bfloat16 *__restrict__ hi,
                                                                 __nv_bfloat16 *__restrict__ lo) {
  __shared__ uint32_t sh[2][TR][TK / 2 + 1];
  __shared__ TapTable tt;
  const int r0 = blockIdx.x * TR;
  const int64_t plane = (int64_t)g.in0 * g.in1 * g.in2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = r0 + lane;
  const bool live = row < rows;
  const float *xb = x;
  Win w = {0, 0, 0, 0};
  if (live) {
    const int img = row / g.P;
    const int p = row - img * g.P;
    xb = x + ((b0 + img) * g.cin + grp * g.cpg) * plane;
    w = make_win(g, p);
  }
  for (int k0 = 0; k0 < kp; k0 += TK) {
    __syncthreads();  // the previous tile's words and taps are consumed
    fill_taps(tt, g, k0);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < TK / 2 / 8; i++) {
      const int kp2 = warp + 8 * i;  // k pair
      float v[2] = {0.f, 0.f};
      if (live) {
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int off = tap_of(tt, g, w, 2 * kp2 + e);
          if (off >= 0) v[e] = __ldg(xb + off);
        }
      }
      split_bf16x2(v[0], v[1], sh[0][lane][kp2], sh[1][lane][kp2]);
    }
    __syncthreads();
    // Warp w writes rows 4w .. 4w+3: 32 words (128 bytes) per row and plane.
#pragma unroll
    for (int j = 0; j < TR / 8; j++) {
      const int rr = warp * (TR / 8) + j;
      if (r0 + rr < rows) {
        const int64_t o = (int64_t)(r0 + rr) * kp + k0 + 2 * lane;
        *reinterpret_cast<uint32_t *>(hi + o) = sh[0][rr][lane];
        *reinterpret_cast<uint32_t *>(lo + o) = sh[1][rr][lane];
      }
    }
  }
}

// int8 / uint8 rows [rows][kg]: a CTA owns 32 pixels (lane = pixel) and walks
// kg in tiles of 64 k; each thread packs four consecutive k into a word (odd
// shared pitch), then the rows go out as 64-byte segments. VEC: kg % 4 == 0
// (word stores).
template <bool VEC>
__global__ void __launch_bounds__(256) conv_im2col_i8_kernel(const uint8_t *__restrict__ x, const Geo32 g,
                                                             int64_t grp, int64_t b0, int rows, int kg,
                                                             const uint8_t *xzp, uint8_t *__restrict__ out) {
  __shared__ uint32_t sh[TR][TK / 4 + 1];
  __shared__ TapTable tt;
  const int r0 = blockIdx.x * TR;
  const int64_t plane = (int64_t)g.in0 * g.in1 * g.in2;
  const uint32_t zp = xzp ? *xzp : 0u;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = r0 + lane;
  const bool live = row < rows;
  const uint8_t *xb = x;
  Win w = {0, 0, 0, 0};
  if (live) {
    const int img = row / g.P;
    const int p = row - img * g.P;
    xb = x + ((b0 + img) * g.cin + grp * g.cpg) * plane;
    w = make_win(g, p);
  }
  for (int k0 = 0; k0 < kg; k0 += TK) {
    __syncthreads();
    fill_taps(tt, g, k0);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < TK / 4 / 8; i++) {
      const int k4 = warp + 8 * i;  // k quad
      uint32_t word = 0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        uint32_t v = zp;
        if (live) {
          const int off = tap_of(tt, g, w, 4 * k4 + e);
          if (off >= 0) v = __ldg(xb + off);
        }
        word |= v << (8 * e);
      }
      sh[lane][k4] = word;
    }
    __syncthreads();
    // 32 rows x 16 words: thread t writes word t & 15 of rows (t >> 4) and (t >> 4) + 16.
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int rr = (threadIdx.x >> 4) + 16 * j, wd = threadIdx.x & 15;
      if (r0 + rr >= rows) continue;
      const uint32_t word = sh[rr][wd];
      const int k = k0 + 4 * wd;
      uint8_t *dst = out + (int64_t)(r0 + rr) * kg + k;
      if (VEC) {
        if (k < kg) *reinterpret_cast<uint32_t *>(dst) = word;
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (k + e < kg) dst[e] = (uint8_t)(word >> (8 * e));
      }
    }
  }
}

// One output element per thread, pixels fastest; the taps are walked in
// (c, kz, ky, kx) order by nested loops.
__global__ void __launch_bounds__(256) conv_direct_double_kernel(const float *__restrict__ x,
                                                                 const float *__restrict__ wt,
                                                                 const float *__restrict__ bias, const Geo32 g,
                                                                 int64_t n, int pad_taps, float *__restrict__ y) {
  const int64_t total = n * g.m * (int64_t)g.P;
  const int64_t plane = (int64_t)g.in0 * g.in1 * g.in2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % g.P);
    const int64_t r = i / g.P;
    const int om = (int)(r % g.m);
    const int64_t b = r / g.m;
    const int grp = om / g.mpg;
    const float *xb = x + (b * g.cin + (int64_t)grp * g.cpg) * plane;
    const Win w = make_win(g, p);
    double acc = bias ? (double)__ldg(bias + om) : 0.0;
    const float *wp = wt + om;
    for (int c = 0; c < g.cpg; c++)
      for (int kz = 0; kz < g.k0; kz++)
        for (int ky = 0; ky < g.k1; ky++)
          for (int kx = 0; kx < g.k2; kx++, wp += g.m) {
            const int dz = kz * g.d0, dy = ky * g.d1, dx = kx * g.d2;
            const int off = tap_at(g, w, ((c * g.in0 + dz) * g.in1 + dy) * g.in2 + dx, dz, dy, dx);
            const double wv = (double)__ldg(wp);
            // float x float is exact in double, so fma is the reference's acc += x * w.
            if (off >= 0) acc = fma((double)__ldg(xb + off), wv, acc);
            else if (pad_taps) acc = fma(0.0, wv, acc);
          }
    y[i] = __double2float_rn(acc);
  }
}

// z [rows][mpg] -> NC[D]HW through a 32 x 32 shared-memory transpose: reads
// run along channels, writes along pixels.
template <bool REQ, bool S8>
__global__ void __launch_bounds__(256) conv_scatter_kernel(const int32_t *__restrict__ z, const Geo32 g, int64_t grp,
                                                           int64_t b0, int64_t rows, int32_t *__restrict__ y32,
                                                           uint8_t *__restrict__ yq, const ConvRequant rq) {
  __shared__ int32_t t[32][33];
  const int64_t r0 = (int64_t)blockIdx.x * 32;
  const int j0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int rr = ty; rr < 32; rr += 8) {
    const int64_t row = r0 + rr;
    const int j = j0 + tx;
    if (row < rows && j < g.mpg) t[rr][tx] = z[row * g.mpg + j];
  }
  __syncthreads();
  for (int jj = ty; jj < 32; jj += 8) {
    const int j = j0 + jj;
    const int64_t row = r0 + tx;
    if (j >= g.mpg || row >= rows) continue;
    const int64_t img = row / g.P;
    const int64_t p = row - img * g.P;
    const int ch = (int)grp * g.mpg + j;
    const int64_t o = ((b0 + img) * g.m + ch) * (int64_t)g.P + p;
    const int32_t acc = t[tx][jj];
    if (!REQ) {
      y32[o] = acc;
    } else {
      const int64_t sum = (int64_t)acc + (rq.bias ? (int64_t)__ldg(rq.bias + ch) : 0);
      // (x_scale * w_scale) / y_scale, left to right in double (:370).
      const double mult = __ddiv_rn(__dmul_rn(rq.xs, (double)__ldg(rq.ws + (rq.ws_len == 1 ? 0 : ch))), rq.ys);
      double v = __dmul_rn((double)sum, mult);
      // Values beyond +-2^40 clamp to lo / hi either way.
      v = fmin(fmax(v, -1099511627776.0), 1099511627776.0);
      int64_t q = __double2ll_rn(v) + rq.y_zp;  // round half to even
      q = q < rq.lo ? rq.lo : (q > rq.hi ? rq.hi : q);
      yq[o] = S8 ? (uint8_t)(int8_t)q : (uint8_t)q;
    }
  }
}

// ConvTranspose, GEMM path: one thread per output element of the group.
__global__ void __launch_bounds__(256) conv_transpose_col2im_kernel(const float *__restrict__ prod, const ConvTGeom g,
                                                                    int64_t grp, const float *__restrict__ bias,
                                                                    float *__restrict__ y) {
  const int64_t out_hw = g.out[1] * g.out[2], in_hw = g.in[1] * g.in[2];
  const int64_t total = g.mpg * out_hw;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t mm = i / out_hw, r = i - mm * out_hw;
    const int64_t oh = r / g.out[2], ow = r - oh * g.out[2];
    float acc = 0.f;
    for (int64_t kh = 0; kh < g.k[1]; kh++) {
      const int64_t nh = oh + g.pad[1] - kh * g.dil[1];
      if (nh < 0 || nh % g.st[1]) continue;
      const int64_t ih = nh / g.st[1];
      if (ih >= g.in[1]) continue;
      for (int64_t kw = 0; kw < g.k[2]; kw++) {
        const int64_t nw = ow + g.pad[2] - kw * g.dil[2];
        if (nw < 0 || nw % g.st[2]) continue;
        const int64_t iw = nw / g.st[2];
        if (iw >= g.in[2]) continue;
        acc = __fadd_rn(acc, __ldg(prod + ((mm * g.k[1] + kh) * g.k[2] + kw) * in_hw + ih * g.in[2] + iw));
      }
    }
    const int64_t om = grp * g.mpg + mm;
    if (bias) acc = __fadd_rn(acc, __ldg(bias + om));
    y[om * out_hw + r] = acc;
  }
}

// ConvTranspose, generic path: one thread per output element (b, om, o).
// For a fixed output, input position i along an axis pairs with the single
// tap k = (o + pad - i * stride) / dilation, so walking k downwards walks i
// upwards: the loops visit (c, i0, i1, i2) in the reference's order.
__global__ void __launch_bounds__(256) conv_transpose_scatter_kernel(const float *__restrict__ x,
                                                                     const float *__restrict__ w,
                                                                     const float *__restrict__ bias, const ConvTGeom g,
                                                                     float *__restrict__ y) {
  const int64_t out_n = g.out[0] * g.out[1] * g.out[2];
  const int64_t kvol = g.k[0] * g.k[1] * g.k[2];
  const int64_t total = g.n * g.m * out_n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i % out_n, bm = i / out_n;
    const int64_t om = bm % g.m, b = bm / g.m;
    const int64_t grp = om / g.mpg, mm = om - grp * g.mpg;
    const int64_t o2 = r % g.out[2], o1 = (r / g.out[2]) % g.out[1], o0 = r / (g.out[1] * g.out[2]);
    float acc = 0.f;
    for (int64_t c = grp * g.cpg; c < (grp + 1) * g.cpg; c++) {
      const float *xc = x + (b * g.cin + c) * g.in[0] * g.in[1] * g.in[2];
      const float *wc = w + (c * g.mpg + mm) * kvol;
      for (int64_t k0 = g.k[0] - 1; k0 >= 0; k0--) {
        const int64_t n0 = o0 + g.pad[0] - k0 * g.dil[0];
        if (n0 < 0 || n0 % g.st[0]) continue;
        const int64_t i0 = n0 / g.st[0];
        if (i0 >= g.in[0]) continue;
        for (int64_t k1 = g.k[1] - 1; k1 >= 0; k1--) {
          const int64_t n1 = o1 + g.pad[1] - k1 * g.dil[1];
          if (n1 < 0 || n1 % g.st[1]) continue;
          const int64_t i1 = n1 / g.st[1];
          if (i1 >= g.in[1]) continue;
          for (int64_t k2 = g.k[2] - 1; k2 >= 0; k2--) {
            const int64_t n2 = o2 + g.pad[2] - k2 * g.dil[2];
            if (n2 < 0 || n2 % g.st[2]) continue;
            const int64_t i2 = n2 / g.st[2];
            if (i2 >= g.in[2]) continue;
            const float v = __ldg(xc + (i0 * g.in[1] + i1) * g.in[2] + i2);
            if (v == 0.f) continue;
            // float x float is exact in double; one double add, then float32.
            const double p = __dmul_rn((double)v, (double)__ldg(wc + (k0 * g.k[1] + k1) * g.k[2] + k2));
            acc = __double2float_rn(__dadd_rn((double)acc, p));
          }
        }
      }
    }
    if (bias) acc = __fadd_rn(acc, __ldg(bias + om));
    y[i] = acc;
  }
}

unsigned grid_for(int64_t total) {
  const int64_t want = (total + 255) / 256;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)device_sm_count() * 16));
}

}  // namespace

void launch_conv_im2col_f32(const float *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, float *cols,
                            cudaStream_t s) {
  if (nb <= 0 || g.K <= 0 || g.P <= 0) return;
  B2M_REQUIRE(nb <= 65535 && (g.K + TK - 1) / TK <= 65535, B2M_ERR_UNSUPPORTED, "Conv: panel too large");
  const dim3 grid((unsigned)((g.P + 255) / 256), (unsigned)((g.K + TK - 1) / TK), (unsigned)nb);
  conv_im2col_f32_kernel<<<grid, 256, 0, s>>>(x, geo32(g), grp, b0, cols);
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_im2col_planes(const float *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int64_t kp,
                               void *hi, void *lo, cudaStream_t s) {
  const int64_t rows = nb * g.P;
  if (rows <= 0) return;
  B2M_REQUIRE(kp % TK == 0 && rows < INT32_MAX && kp < INT32_MAX, B2M_ERR_UNSUPPORTED, "Conv: panel too large");
  conv_im2col_planes_kernel<<<(unsigned)((rows + TR - 1) / TR), 256, 0, s>>>(
      x, geo32(g), grp, b0, (int)rows, (int)kp, static_cast<__nv_bfloat16 *>(hi), static_cast<__nv_bfloat16 *>(lo));
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_im2col_i8(const void *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int64_t kg,
                           const void *xzp, uint8_t *rows_out, cudaStream_t s) {
  const int64_t rows = nb * g.P;
  if (rows <= 0) return;
  B2M_REQUIRE(rows < INT32_MAX && kg < INT32_MAX, B2M_ERR_UNSUPPORTED, "Conv: panel too large");
  const unsigned grid = (unsigned)((rows + TR - 1) / TR);
  const uint8_t *xb = static_cast<const uint8_t *>(x);
  const uint8_t *zp = static_cast<const uint8_t *>(xzp);
  if (kg % 4 == 0)
    conv_im2col_i8_kernel<true><<<grid, 256, 0, s>>>(xb, geo32(g), grp, b0, (int)rows, (int)kg, zp, rows_out);
  else
    conv_im2col_i8_kernel<false><<<grid, 256, 0, s>>>(xb, geo32(g), grp, b0, (int)rows, (int)kg, zp, rows_out);
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_direct_double(const float *x, const float *wt, const float *bias, const ConvGeom &g, int pad_taps,
                               float *y, cudaStream_t s) {
  const int64_t total = g.n * g.m * g.P;
  if (total <= 0) return;
  conv_direct_double_kernel<<<grid_for(total), 256, 0, s>>>(x, wt, bias, geo32(g), g.n, pad_taps, y);
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_scatter(const int32_t *z, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int32_t *y32,
                         void *yq, const ConvRequant &rq, cudaStream_t s) {
  const int64_t rows = nb * g.P;
  if (rows <= 0 || g.mpg <= 0) return;
  B2M_REQUIRE((rows + 31) / 32 <= INT32_MAX && (g.mpg + 31) / 32 <= 65535, B2M_ERR_UNSUPPORTED,
              "Conv: output too large");
  dim3 grid((unsigned)((rows + 31) / 32), (unsigned)((g.mpg + 31) / 32));
  const Geo32 g32 = geo32(g);
  uint8_t *q = static_cast<uint8_t *>(yq);
  if (!yq) conv_scatter_kernel<false, false><<<grid, 256, 0, s>>>(z, g32, grp, b0, rows, y32, q, rq);
  else if (rq.lo < 0) conv_scatter_kernel<true, true><<<grid, 256, 0, s>>>(z, g32, grp, b0, rows, y32, q, rq);
  else conv_scatter_kernel<true, false><<<grid, 256, 0, s>>>(z, g32, grp, b0, rows, y32, q, rq);
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_transpose_col2im(const float *prod, const ConvTGeom &g, int64_t grp, const float *bias, float *y,
                                  cudaStream_t s) {
  const int64_t total = g.mpg * g.out[1] * g.out[2];
  if (total <= 0) return;
  conv_transpose_col2im_kernel<<<grid_for(total), 256, 0, s>>>(prod, g, grp, bias, y);
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_transpose_scatter(const float *x, const float *w, const float *bias, const ConvTGeom &g, float *y,
                                   cudaStream_t s) {
  const int64_t total = g.n * g.m * g.out[0] * g.out[1] * g.out[2];
  if (total <= 0) return;
  conv_transpose_scatter_kernel<<<grid_for(total), 256, 0, s>>>(x, w, bias, g, y);
  B2M_CUDA(cudaGetLastError());
}
