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

// Element offset of tap k of pixel p inside one image's group-channel block
// (channel c of the group at plane offset c * in0*in1*in2), or -1 when the
// tap falls in the padding.
__device__ __forceinline__ int64_t tap_offset(const Geo32 &g, int k, int p) {
  const int kvol = g.k0 * g.k1 * g.k2;
  const int c = k / kvol, t = k - c * kvol;
  const int kz = t / (g.k1 * g.k2), ky = (t / g.k2) % g.k1, kx = t % g.k2;
  const int oz = p / (g.o1 * g.o2), oy = (p / g.o2) % g.o1, ox = p % g.o2;
  const int iz = oz * g.s0 - g.p0 + kz * g.d0;
  const int iy = oy * g.s1 - g.p1 + ky * g.d1;
  const int ix = ox * g.s2 - g.p2 + kx * g.d2;
  if (iz < 0 || iz >= g.in0 || iy < 0 || iy >= g.in1 || ix < 0 || ix >= g.in2) return -1;
  return (((int64_t)c * g.in0 + iz) * g.in1 + iy) * g.in2 + ix;
}

// fp32 panel [nb][K][P]; consecutive threads take consecutive pixels, so a
// stride-1 row of taps reads and writes contiguous memory.
__global__ void __launch_bounds__(256) conv_im2col_f32_kernel(const float *__restrict__ x, const Geo32 g, int64_t grp,
                                                              int64_t b0, int64_t nb, float *__restrict__ cols) {
  const int64_t total = nb * g.K * (int64_t)g.P;
  const int64_t plane = (int64_t)g.in0 * g.in1 * g.in2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % g.P);
    const int64_t r = i / g.P;
    const int k = (int)(r % g.K);
    const int64_t b = b0 + r / g.K;
    const int64_t off = tap_offset(g, k, p);
    cols[i] = off < 0 ? 0.f : __ldg(x + (b * g.cin + grp * g.cpg) * plane + off);
  }
}

constexpr int TR = 32;  // panel rows (pixels) per tile
constexpr int TK = 64;  // reduction columns per tile

// bf16 split planes [rows][kp]: a tile of 32 pixels x 64 k is gathered with
// pixels along the warp (coalesced reads), split, transposed through shared
// memory and stored as 128-byte row segments of each plane.
__global__ void __launch_bounds__(256) conv_im2col_planes_kernel(const float *__restrict__ x, const Geo32 g,
                                                                 int64_t grp, int64_t b0, int64_t rows, int64_t kp,
                                                                 __nv_bfloat16 *__restrict__ hi,
                                                                 __nv_bfloat16 *__restrict__ lo) {
  __shared__ __align__(16) __nv_bfloat16 sh[2][TR][TK + 8];
  const int64_t r0 = (int64_t)blockIdx.x * TR;
  const int k0 = blockIdx.y * TK;
  const int64_t plane = (int64_t)g.in0 * g.in1 * g.in2;
#pragma unroll
  for (int i = 0; i < (TR * TK) / 256; i++) {
    const int e = threadIdx.x + 256 * i;
    const int kk = e / TR, r = e % TR;
    const int64_t row = r0 + r;
    const int k = k0 + kk;
    float v = 0.f;
    if (row < rows && k < g.K) {
      const int64_t img = row / g.P;
      const int p = (int)(row - img * g.P);
      const int64_t off = tap_offset(g, k, p);
      if (off >= 0) v = __ldg(x + ((b0 + img) * g.cin + grp * g.cpg) * plane + off);
    }
    split_bf16(v, sh[0][r][kk], sh[1][r][kk]);
  }
  __syncthreads();
  // 32 rows x 8 uint4 per plane.
  const int r = threadIdx.x >> 3, q = threadIdx.x & 7;
  const int64_t row = r0 + r;
  if (row < rows) {
    const int64_t o = row * kp + k0 + 8 * q;
    *reinterpret_cast<uint4 *>(hi + o) = *reinterpret_cast<const uint4 *>(&sh[0][r][8 * q]);
    *reinterpret_cast<uint4 *>(lo + o) = *reinterpret_cast<const uint4 *>(&sh[1][r][8 * q]);
  }
}

// int8 / uint8 rows [rows][kg]; VEC stores 16-byte segments (kg % 16 == 0).
template <bool VEC>
__global__ void __launch_bounds__(256) conv_im2col_i8_kernel(const uint8_t *__restrict__ x, const Geo32 g,
                                                             int64_t grp, int64_t b0, int64_t rows, int64_t kg,
                                                             const uint8_t *xzp, uint8_t *__restrict__ out) {
  __shared__ __align__(16) uint8_t sh[TR][TK + 16];
  const int64_t r0 = (int64_t)blockIdx.x * TR;
  const int k0 = blockIdx.y * TK;
  const int64_t plane = (int64_t)g.in0 * g.in1 * g.in2;
  const uint8_t zp = xzp ? *xzp : (uint8_t)0;
#pragma unroll
  for (int i = 0; i < (TR * TK) / 256; i++) {
    const int e = threadIdx.x + 256 * i;
    const int kk = e / TR, r = e % TR;
    const int64_t row = r0 + r;
    const int k = k0 + kk;
    uint8_t v = zp;
    if (row < rows && k < g.K) {
      const int64_t img = row / g.P;
      const int p = (int)(row - img * g.P);
      const int64_t off = tap_offset(g, k, p);
      if (off >= 0) v = __ldg(x + ((b0 + img) * g.cin + grp * g.cpg) * plane + off);
    }
    sh[r][kk] = v;
  }
  __syncthreads();
  if (VEC) {
    if (threadIdx.x < TR * (TK / 16)) {
      const int r = threadIdx.x >> 2, q = threadIdx.x & 3;
      const int64_t row = r0 + r;
      const int64_t k = k0 + 16 * q;
      if (row < rows && k < kg)
        *reinterpret_cast<uint4 *>(out + row * kg + k) = *reinterpret_cast<const uint4 *>(&sh[r][16 * q]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < (TR * TK) / 256; i++) {
      const int e = threadIdx.x + 256 * i;
      const int r = e / TK, kk = e % TK;
      const int64_t row = r0 + r;
      const int64_t k = k0 + kk;
      if (row < rows && k < kg) out[row * kg + k] = sh[r][kk];
    }
  }
}

// One output element per thread, pixels fastest.
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
    double acc = bias ? (double)__ldg(bias + om) : 0.0;
    for (int k = 0; k < g.K; k++) {
      const int64_t off = tap_offset(g, k, p);
      const double wv = (double)__ldg(wt + (int64_t)k * g.m + om);
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
                                                           uint8_t *__restrict__ yq, const double *__restrict__ mult,
                                                           const int32_t *__restrict__ bias, int32_t y_zp, int32_t lo,
                                                           int32_t hi) {
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
      const int64_t sum = (int64_t)acc + (bias ? (int64_t)__ldg(bias + ch) : 0);
      double v = (double)sum * __ldg(mult + ch);
      // Values beyond +-2^40 clamp to lo / hi either way.
      v = fmin(fmax(v, -1099511627776.0), 1099511627776.0);
      int64_t q = __double2ll_rn(v) + y_zp;  // round half to even
      q = q < lo ? lo : (q > hi ? hi : q);
      yq[o] = S8 ? (uint8_t)(int8_t)q : (uint8_t)q;
    }
  }
}

unsigned grid_for(int64_t total) {
  const int64_t want = (total + 255) / 256;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)device_sm_count() * 16));
}

}  // namespace

void launch_conv_im2col_f32(const float *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, float *cols,
                            cudaStream_t s) {
  const int64_t total = nb * g.K * g.P;
  if (total <= 0) return;
  conv_im2col_f32_kernel<<<grid_for(total), 256, 0, s>>>(x, geo32(g), grp, b0, nb, cols);
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_im2col_planes(const float *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int64_t kp,
                               void *hi, void *lo, cudaStream_t s) {
  const int64_t rows = nb * g.P;
  if (rows <= 0) return;
  B2M_REQUIRE(kp % TK == 0 && (rows + TR - 1) / TR <= INT32_MAX && kp / TK <= 65535, B2M_ERR_UNSUPPORTED,
              "Conv: panel too large");
  dim3 grid((unsigned)((rows + TR - 1) / TR), (unsigned)(kp / TK));
  conv_im2col_planes_kernel<<<grid, 256, 0, s>>>(x, geo32(g), grp, b0, rows, kp, static_cast<__nv_bfloat16 *>(hi),
                                                 static_cast<__nv_bfloat16 *>(lo));
  B2M_CUDA(cudaGetLastError());
}

void launch_conv_im2col_i8(const void *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int64_t kg,
                           const void *xzp, uint8_t *rows_out, cudaStream_t s) {
  const int64_t rows = nb * g.P;
  if (rows <= 0) return;
  const int64_t kt = (kg + TK - 1) / TK;
  B2M_REQUIRE((rows + TR - 1) / TR <= INT32_MAX && kt <= 65535, B2M_ERR_UNSUPPORTED, "Conv: panel too large");
  dim3 grid((unsigned)((rows + TR - 1) / TR), (unsigned)kt);
  const uint8_t *xb = static_cast<const uint8_t *>(x);
  const uint8_t *zp = static_cast<const uint8_t *>(xzp);
  if (kg % 16 == 0)
    conv_im2col_i8_kernel<true><<<grid, 256, 0, s>>>(xb, geo32(g), grp, b0, rows, kg, zp, rows_out);
  else
    conv_im2col_i8_kernel<false><<<grid, 256, 0, s>>>(xb, geo32(g), grp, b0, rows, kg, zp, rows_out);
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
                         void *yq, const double *mult, const int32_t *bias, int32_t y_zp, int32_t lo, int32_t hi,
                         cudaStream_t s) {
  const int64_t rows = nb * g.P;
  if (rows <= 0 || g.mpg <= 0) return;
  B2M_REQUIRE((rows + 31) / 32 <= INT32_MAX && (g.mpg + 31) / 32 <= 65535, B2M_ERR_UNSUPPORTED,
              "Conv: output too large");
  dim3 grid((unsigned)((rows + 31) / 32), (unsigned)((g.mpg + 31) / 32));
  const Geo32 g32 = geo32(g);
  uint8_t *q = static_cast<uint8_t *>(yq);
  if (!yq) conv_scatter_kernel<false, false><<<grid, 256, 0, s>>>(z, g32, grp, b0, rows, y32, q, mult, bias, y_zp, lo, hi);
  else if (lo < 0) conv_scatter_kernel<true, true><<<grid, 256, 0, s>>>(z, g32, grp, b0, rows, y32, q, mult, bias, y_zp, lo, hi);
  else conv_scatter_kernel<true, false><<<grid, 256, 0, s>>>(z, g32, grp, b0, rows, y32, q, mult, bias, y_zp, lo, hi);
  B2M_CUDA(cudaGetLastError());
}
