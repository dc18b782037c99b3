// Device-resident glue for the MatMul chains of a transformer layer, so a
// chain never round-trips through host memory between its MatMuls:
//   RMSNorm (+ fused residual add)   opRMSNorm, onnx_ops.dart:1771; fused
//                                    SkipSimplifiedLayerNormalization,
//                                    onnx_graph.dart:1793
//   LayerNormalization (+ residual)  opLayerNormalization, onnx_ops.dart:1666
//   SwiGLU silu(gate) * up           the Sigmoid/Mul pair of the MLP
//   erf GELU                         opGelu, onnx_ops.dart:706
//   Gather of embedding rows         opGather
//   ArgMax over the last axis        opArgMinMax, onnx_ops.dart (first max wins)
//   GroupQueryAttention              opGroupQueryAttention, onnx_ops.dart:1844
//                                    with rotary (opRotaryEmbedding, :2659)
// The reductions accumulate in double where the reference does (norm
// statistics, softmax sums); elementwise math is fp32. The attention keeps its
// K/V in a caller-owned cache [B][KVH][CAP][D] and reads the number of cached
// positions from device memory, so a decode step replays as a CUDA graph.
#include <algorithm>
#include <cfloat>

#include <cuda_bf16.h>

#include "b2m_internal.cuh"
#include "tc_common.cuh"

// Every glue kernel triggers programmatic dependent launch at entry: the
// next kernel of the stream, when it is launched that way (the GEMMs and
// GEMVs are), starts its weight-side prologue under this one and waits for
// this grid (griddepcontrol.wait) before it reads or writes anything this
// grid touches.
namespace {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row of length D. With `skip`, the row is x + skip (stored to
// `sum_out` when given) before normalising: y = s * inv * gamma, inv =
// 1/sqrt(mean(s^2) + eps) with the mean accumulated in double.
// Rows are laid out as groups of `per` rows of D (offset g*gstride + i*D for
// row r = g*per + i); contiguous rows have per = rows, gstride = 0.
// RMSNorm / LayerNorm, one warp per row. The reference reduces in double;
// double arithmetic is a small fraction of the fp32 rate on this part, so the
// row (VPL values per lane, all loads in flight together) is reduced in fp32
// (per-lane partial sums, then a warp tree: relative error ~1e-6 for rows of
// a few thousand) and only the per-row factor is formed in double. Outputs
// may overwrite the input in place.
template <int VPL>
__device__ __forceinline__ void norm_load(const float *xr, const float *sr, int D, int lane, float (&v)[VPL]) {
#pragma unroll
  for (int i = 0; i < VPL; i++) {
    const int j = lane + 32 * i;
    v[i] = j < D ? (sr ? xr[j] + sr[j] : xr[j]) : 0.f;
  }
}

template <int VPL>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *x, const float *skip, const float *__restrict__ gamma,
                                                      float *y, float *sum_out, int64_t rows, int D, double eps,
                                                      int64_t per, int64_t gstride, int64_t gamma_rs) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const int64_t off = (r / per) * gstride + (r % per) * D;
  const float *gm = gamma + (r % per) * gamma_rs;  // per-row gains (gamma_rs = D) or one row (0)
  float v[VPL];
  norm_load<VPL>(x + off, skip ? skip + off : nullptr, D, lane, v);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; i++) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum_f(ss);
  const float inv = (float)(1.0 / sqrt((double)ss / D + eps));
#pragma unroll
  for (int i = 0; i < VPL; i++) {
    const int j = lane + 32 * i;
    if (j < D) {
      if (sum_out) sum_out[off + j] = v[i];
      y[off + j] = v[i] * inv * gm[j];
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(256) layernorm_kernel(const float *x, const float *skip,
                                                        const float *__restrict__ gamma, const float *__restrict__ beta,
                                                        float *y, float *sum_out, int64_t rows, int D, double eps) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  float v[VPL];
  norm_load<VPL>(x + r * D, skip ? skip + r * D : nullptr, D, lane, v);
  float s1 = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; i++) s1 += v[i];
  const float mean = warp_sum_f(s1) / (float)D;
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; i++) {
    const float d = lane + 32 * i < D ? v[i] - mean : 0.f;
    s2 = fmaf(d, d, s2);
  }
  const float inv = (float)(1.0 / sqrt((double)warp_sum_f(s2) / D + eps));
#pragma unroll
  for (int i = 0; i < VPL; i++) {
    const int j = lane + 32 * i;
    if (j < D) {
      if (sum_out) sum_out[r * D + j] = v[i];
      y[r * D + j] = (v[i] - mean) * inv * gamma[j] + (beta ? beta[j] : 0.f);
    }
  }
}

// Four values as f16, round to nearest (the rounding of f32_to_f16_rows, so a
// producer's f16 copy equals what the GEMM's own conversion would form).
__device__ __forceinline__ void store_f16x4(__half *p, float4 v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t *>(&a);
  u.y = *reinterpret_cast<const uint32_t *>(&b);
  *reinterpret_cast<uint2 *>(p) = u;
}

// Four values as bf16 hi / lo planes (split_bf16x2 pairs, the split of
// f32_split_rows, so a producer's planes equal what the FAST GEMM's own split
// forms).
__device__ __forceinline__ void store_split4(__nv_bfloat16 *p0, __nv_bfloat16 *p1, int64_t i, float4 v) {
  uint2 h, l;
  b2m::split_bf16x2(v.x, v.y, h.x, l.x);
  b2m::split_bf16x2(v.z, v.w, h.y, l.y);
  *reinterpret_cast<uint2 *>(p0 + i) = h;
  *reinterpret_cast<uint2 *>(p1 + i) = l;
}

// Warp per row with float4 loads (D % 4 == 0, 16-byte aligned rows): lane
// takes float4 chunks lane + 32 i. Half the load instructions of the scalar
// form and twice the bytes per request (BERT LayerNorm 4096 x 768: 6.5 us
// against 12 us).
template <int V4, bool LN>
__global__ void __launch_bounds__(256) norm_warp4_kernel(const float *x, const float *skip,
                                                         const float *__restrict__ gamma,
                                                         const float *__restrict__ beta, float *y, float *sum_out,
                                                         int64_t rows, int D, double eps, int64_t per,
                                                         int64_t gstride, int64_t gamma_rs, __half *y16,
                                                         __nv_bfloat16 *p0, __nv_bfloat16 *p1) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const int64_t off = (r / per) * gstride + (r % per) * D;
  const float *gm = gamma + (r % per) * gamma_rs;  // per-row gains (gamma_rs = D) or one row (0)
  const int d4 = D >> 2;
  const float4 *xr = reinterpret_cast<const float4 *>(x + off);
  const float4 *sr = skip ? reinterpret_cast<const float4 *>(skip + off) : nullptr;
  float4 v[V4];
#pragma unroll
  for (int i = 0; i < V4; i++) {
    const int j = lane + 32 * i;
    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < d4) {
      v[i] = xr[j];
      if (sr) {
        const float4 t = sr[j];
        v[i].x += t.x, v[i].y += t.y, v[i].z += t.z, v[i].w += t.w;
      }
    }
  }
  float mean = 0.f;
  if (LN) {
    float s1 = 0.f;
#pragma unroll
    for (int i = 0; i < V4; i++) s1 += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    mean = warp_sum_f(s1) / (float)D;
  }
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < V4; i++)
    if (lane + 32 * i < d4) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      s2 = fmaf(a, a, fmaf(b, b, fmaf(c, c, fmaf(d, d, s2))));
    }
  const float inv = (float)(1.0 / sqrt((double)warp_sum_f(s2) / D + eps));
  const float4 *g4 = reinterpret_cast<const float4 *>(gm);
  const float4 *b4 = beta ? reinterpret_cast<const float4 *>(beta) : nullptr;
#pragma unroll
  for (int i = 0; i < V4; i++) {
    const int j = lane + 32 * i;
    if (j < d4) {
      if (sum_out) reinterpret_cast<float4 *>(sum_out + off)[j] = v[i];
      const float4 g = g4[j];
      const float4 bb = b4 ? b4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 o = make_float4((v[i].x - mean) * inv * g.x + bb.x, (v[i].y - mean) * inv * g.y + bb.y,
                                   (v[i].z - mean) * inv * g.z + bb.z, (v[i].w - mean) * inv * g.w + bb.w);
      if (y) reinterpret_cast<float4 *>(y + off)[j] = o;
      if (y16) store_f16x4(y16 + off + 4 * j, o);
      if (p0) store_split4(p0, p1, off + 4 * j, o);
    }
  }
}

// One CTA per row for few rows (a decode step's 64 tokens): float4 loads
// spread over up to 256 threads instead of one warp walking the row, which
// is what a handful of rows on a handful of SMs needs (64 x 1024: 1.7 us
// against 8 us warp-per-row). Rows of D floats at offsets
// (r / per) * gstride + (r % per) * D, D % 4 == 0 and 16-byte aligned
// operands; NV4 float4 per thread (D <= 1024 * NV4).
template <int NV4, bool LN>
__global__ void __launch_bounds__(256) norm_row_cta_kernel(const float *x, const float *skip,
                                                           const float *__restrict__ gamma,
                                                           const float *__restrict__ beta, float *y, float *sum_out,
                                                           int D, double eps, int64_t per, int64_t gstride, int64_t gamma_rs,
                                                           __half *y16, __nv_bfloat16 *p0, __nv_bfloat16 *p1) {
  b2m::pdl_launch_dependents();
  const int64_t r = blockIdx.x;
  const int64_t off = (r / per) * gstride + (r % per) * D;
  const float *gm = gamma + (r % per) * gamma_rs;  // per-row gains (gamma_rs = D) or one row (0)
  const int d4 = D >> 2, tid = threadIdx.x, nt = blockDim.x;
  const float4 *xr = reinterpret_cast<const float4 *>(x + off);
  const float4 *sr = skip ? reinterpret_cast<const float4 *>(skip + off) : nullptr;
  float4 v[NV4];
#pragma unroll
  for (int i = 0; i < NV4; i++) {
    const int j = tid + nt * i;
    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < d4) {
      v[i] = xr[j];
      if (sr) {
        const float4 t = sr[j];
        v[i].x += t.x, v[i].y += t.y, v[i].z += t.z, v[i].w += t.w;
      }
    }
  }
  __shared__ float red[8];
  auto block_sum = [&](float t) {
    t = warp_sum_f(t);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = t;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < (nt + 31) / 32; w++) tot += red[w];
    return tot;
  };
  float mean = 0.f;
  if (LN) {
    float s1 = 0.f;
#pragma unroll
    for (int i = 0; i < NV4; i++) s1 += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    mean = block_sum(s1) / (float)D;
  }
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < NV4; i++)
    if (tid + nt * i < d4) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      s2 = fmaf(a, a, fmaf(b, b, fmaf(c, c, fmaf(d, d, s2))));
    }
  const float inv = (float)(1.0 / sqrt((double)block_sum(s2) / D + eps));
  const float4 *g4 = reinterpret_cast<const float4 *>(gm);
  const float4 *b4 = beta ? reinterpret_cast<const float4 *>(beta) : nullptr;
#pragma unroll
  for (int i = 0; i < NV4; i++) {
    const int j = tid + nt * i;
    if (j < d4) {
      if (sum_out) reinterpret_cast<float4 *>(sum_out + off)[j] = v[i];
      const float4 g = g4[j];
      const float4 bb = b4 ? b4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 o = make_float4((v[i].x - mean) * inv * g.x + bb.x, (v[i].y - mean) * inv * g.y + bb.y,
                                   (v[i].z - mean) * inv * g.z + bb.z, (v[i].w - mean) * inv * g.w + bb.w);
      if (y) reinterpret_cast<float4 *>(y + off)[j] = o;
      if (y16) store_f16x4(y16 + off + 4 * j, o);
      if (p0) store_split4(p0, p1, off + 4 * j, o);
    }
  }
}

// Launches the CTA-per-row variant when the rows are few and the layout
// allows float4; returns false otherwise.
template <bool LN>
bool launch_norm_rows_cta(const float *x, const float *skip, const float *gamma, const float *beta, float *y,
                          float *sum_out, int64_t rows, int D, double eps, int64_t per, int64_t gstride,
                          int64_t gamma_rs, cudaStream_t s, __half *y16 = nullptr, __nv_bfloat16 *p0 = nullptr,
                          __nv_bfloat16 *p1 = nullptr) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (D % 4 || gstride % 4 || D > 4096 || !al(x) || !al(skip) || !al(gamma) || !al(beta) || !al(y) ||
      !al(sum_out))
    return false;
  if (rows > 4 * (int64_t)b2m::device_sm_count() || rows > 2147483647) {
    // Many rows: a warp per row, float4 loads.
    const unsigned g = (unsigned)((rows + 7) / 8);
    const int v4 = (D / 4 + 31) / 32;
#define B2M_NW4(N) \
  norm_warp4_kernel<N, LN><<<g, 256, 0, s>>>(x, skip, gamma, beta, y, sum_out, rows, D, eps, per, gstride, \
                                              gamma_rs, y16, p0, p1)
    if (v4 <= 1) B2M_NW4(1);
    else if (v4 <= 2) B2M_NW4(2);
    else if (v4 <= 4) B2M_NW4(4);
    else if (v4 <= 6) B2M_NW4(6);
    else if (v4 <= 8) B2M_NW4(8);
    else if (v4 <= 16) B2M_NW4(16);
    else return false;
#undef B2M_NW4
    B2M_CUDA(cudaGetLastError());
    return true;
  }
  const int d4 = D / 4;
  const int nt = std::min(256, (d4 + 31) / 32 * 32);
  const int nv4 = (d4 + nt - 1) / nt;
  const unsigned g = (unsigned)rows;
#define B2M_NRC(N) \
  norm_row_cta_kernel<N, LN><<<g, nt, 0, s>>>(x, skip, gamma, beta, y, sum_out, D, eps, per, gstride, gamma_rs, y16, \
                                               p0, p1)
  if (nv4 <= 1) B2M_NRC(1);
  else if (nv4 <= 2) B2M_NRC(2);
  else B2M_NRC(4);
#undef B2M_NRC
  B2M_CUDA(cudaGetLastError());
  return true;
}

// Rows longer than 32 x 64 values: the same arithmetic streamed from memory.
__global__ void __launch_bounds__(256) rmsnorm_long_kernel(const float *x, const float *skip,
                                                           const float *__restrict__ gamma, float *y, float *sum_out,
                                                           int64_t rows, int D, double eps, int64_t per,
                                                           int64_t gstride, int64_t gamma_rs) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const int64_t off = (r / per) * gstride + (r % per) * D;
  const float *gm = gamma + (r % per) * gamma_rs;  // per-row gains (gamma_rs = D) or one row (0)
  const float *xr = x + off;
  const float *sr = skip ? skip + off : nullptr;
  float ss = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float v = sr ? xr[j] + sr[j] : xr[j];
    ss = fmaf(v, v, ss);
  }
  const float inv = (float)(1.0 / sqrt((double)warp_sum_f(ss) / D + eps));
  for (int j = lane; j < D; j += 32) {
    const float v = sr ? xr[j] + sr[j] : xr[j];
    if (sum_out) sum_out[off + j] = v;
    y[off + j] = v * inv * gm[j];
  }
}

__global__ void __launch_bounds__(256) layernorm_long_kernel(const float *x, const float *skip,
                                                             const float *__restrict__ gamma,
                                                             const float *__restrict__ beta, float *y, float *sum_out,
                                                             int64_t rows, int D, double eps) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const float *xr = x + r * D;
  const float *sr = skip ? skip + r * D : nullptr;
  float s1 = 0.f;
  for (int j = lane; j < D; j += 32) s1 += sr ? xr[j] + sr[j] : xr[j];
  const float mean = warp_sum_f(s1) / (float)D;
  float s2 = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float d = (sr ? xr[j] + sr[j] : xr[j]) - mean;
    s2 = fmaf(d, d, s2);
  }
  const float inv = (float)(1.0 / sqrt((double)warp_sum_f(s2) / D + eps));
  for (int j = lane; j < D; j += 32) {
    const float v = sr ? xr[j] + sr[j] : xr[j];
    if (sum_out) sum_out[r * D + j] = v;
    y[r * D + j] = (v - mean) * inv * gamma[j] + (beta ? beta[j] : 0.f);
  }
}

// y = silu(gate) * up, with gate / up either separate tensors or the two
// halves of one [rows][2*D] tensor (a packed gate|up projection).
using b2m::silu_times;


// Rows over blockIdx.y, columns over x (float4 when VEC: D, both row strides
// and the three pointers 16-byte aligned); no per-element index division.
template <bool VEC>
__global__ void silu_mul_kernel(const float *__restrict__ gate, const float *__restrict__ up, int64_t g_rs,
                                int64_t u_rs, float *y, int64_t rows, int64_t D, __half *y16) {
  b2m::pdl_launch_dependents();
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const float *gr = gate + r * g_rs, *ur = up + r * u_rs;
    float *yr = y + r * D;
    if (VEC) {
      for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < D / 4; c += step) {
        const float4 g = reinterpret_cast<const float4 *>(gr)[c], u = reinterpret_cast<const float4 *>(ur)[c];
        const float4 o =
            make_float4(silu_times(g.x, u.x), silu_times(g.y, u.y), silu_times(g.z, u.z), silu_times(g.w, u.w));
        reinterpret_cast<float4 *>(yr)[c] = o;
        if (y16) store_f16x4(y16 + r * D + 4 * c, o);
      }
    } else {
      for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < D; c += step) yr[c] = silu_times(gr[c], ur[c]);
    }
  }
}

// SwiGLU over the tile-interleaved output of a gate / up projection: row r
// of y holds, per 128-column tile t, the gate columns 64t .. 64t+63 and then
// the matching up columns; act[r][j] = silu(gate j) * up j (fp32 and / or the
// f16 copy). Four columns per thread (I % 64 == 0, 16-byte aligned rows).
__global__ void silu_mul_tiles_kernel(const float *__restrict__ y, int64_t rows, int64_t I, float *act,
                                      __half *act16) {
  b2m::pdl_launch_dependents();
  const int64_t q = I >> 2, n = rows * q;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / q, c4 = (e - r * q) * 4;
    const float *yr = y + r * 2 * I + (c4 >> 6) * 128 + (c4 & 63);
    const float4 g = *reinterpret_cast<const float4 *>(yr), u = *reinterpret_cast<const float4 *>(yr + 64);
    const float4 o =
        make_float4(silu_times(g.x, u.x), silu_times(g.y, u.y), silu_times(g.z, u.z), silu_times(g.w, u.w));
    if (act) reinterpret_cast<float4 *>(act + r * I)[c4 >> 2] = o;
    if (act16) store_f16x4(act16 + r * I + c4, o);
  }
}

__global__ void gelu_kernel(const float *__restrict__ x, float *y, int64_t n) {
  b2m::pdl_launch_dependents();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    y[i] = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
  }
}

// GELU of n values (n % 4 == 0, 16-byte aligned) written as bf16 hi / lo
// planes (and to y when given): the FAST Gemm's A operand for rows of a
// length that is a multiple of 64 (no padding then).
__global__ void gelu_split_kernel(const float *__restrict__ x, float *y, __nv_bfloat16 *p0, __nv_bfloat16 *p1,
                                  int64_t n4) {
  b2m::pdl_launch_dependents();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4 *>(x)[i];
    float4 o;
    o.x = 0.5f * v.x * (1.f + erff(v.x * 0.70710678118654752f));
    o.y = 0.5f * v.y * (1.f + erff(v.y * 0.70710678118654752f));
    o.z = 0.5f * v.z * (1.f + erff(v.z * 0.70710678118654752f));
    o.w = 0.5f * v.w * (1.f + erff(v.w * 0.70710678118654752f));
    if (y) reinterpret_cast<float4 *>(y)[i] = o;
    store_split4(p0, p1, 4 * i, o);
  }
}

// y = a + b, b broadcast over rows when b_rows == 1.
__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b, float *y, int64_t rows, int64_t D,
                           int b_bcast) {
  b2m::pdl_launch_dependents();
  const int64_t total = rows * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = a[i] + b[b_bcast ? i % D : i];
}

// y[r][:] = table[ids[r]][:] (ids int64); out-of-range ids write zeros and
// raise the error word.
__global__ void gather_rows_kernel(const float *__restrict__ table, const int64_t *__restrict__ ids, float *y,
                                   int64_t rows, int64_t V, int64_t D, int32_t *err) {
  b2m::pdl_launch_dependents();
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const int64_t id = ids[r];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && err) b2m::set_dev_error(err, B2M_DEVERR_INDEX);
  for (int64_t j = threadIdx.x; j < D; j += blockDim.x) y[r * D + j] = ok ? table[id * D + j] : 0.f;
}

// Row argmax (first maximum wins; NaN compares false). One CTA per row.
__device__ __forceinline__ bool argmax_better(float v, int64_t i, float bv, int64_t bi) {
  return v > bv || (v == bv && i < bi);
}

// Partial argmax of one chunk of a row: CTA (chunk c, row r) scans
// [c*chunk, (c+1)*chunk) with float4 loads where the row allows, and writes
// (value, index) of its best element (the smallest index among equal maxima;
// NaN never wins; nothing above -FLT_MAX leaves index V).
__global__ void __launch_bounds__(256) argmax_partial_kernel(const float *__restrict__ x, int64_t V, int64_t chunk,
                                                             float *pv, int64_t *pi) {
  const int64_t r = blockIdx.y, c = blockIdx.x;
  const float *xr = x + r * V;
  const int64_t j0 = c * chunk, j1 = min(V, j0 + chunk);
  float best = -FLT_MAX;
  int64_t bi = V;
  const bool vec = ((V & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((chunk & 3) == 0);
  if (vec) {
    for (int64_t j = j0 + 4 * (int64_t)threadIdx.x; j < j1; j += 4 * 256) {
      const float4 q = *reinterpret_cast<const float4 *>(xr + j);
      const float e[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (argmax_better(e[u], j + u, best, bi)) {
          best = e[u];
          bi = j + u;
        }
    }
  } else {
    for (int64_t j = j0 + threadIdx.x; j < j1; j += 256) {
      const float v = xr[j];
      if (argmax_better(v, j, best, bi)) {
        best = v;
        bi = j;
      }
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (argmax_better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[8];
  __shared__ int64_t si[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; w++)
      if (argmax_better(sv[w], si[w], best, bi)) {
        best = sv[w];
        bi = si[w];
      }
    pv[r * gridDim.x + c] = best;
    pi[r * gridDim.x + c] = bi;
  }
}

// One warp per row combines the chunk results (order-independent rule).
__global__ void __launch_bounds__(256) argmax_final_kernel(const float *pv, const int64_t *pi, int nchunk,
                                                           int64_t *out, int64_t rows, int64_t V) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  float best = -FLT_MAX;
  int64_t bi = V;
  for (int c = lane; c < nchunk; c += 32)
    if (argmax_better(pv[r * nchunk + c], pi[r * nchunk + c], best, bi)) {
      best = pv[r * nchunk + c];
      bi = pi[r * nchunk + c];
    }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (argmax_better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) out[r] = bi < V ? bi : 0;
}

// Rotary of one head vector in place (non-interleaved: pairs (i, i + half);
// interleaved: pairs (2i, 2i+1)), positions index the cos/sin rows.
__device__ __forceinline__ void rotate_head(float *v, const float *cos, const float *sin, int64_t pos, int half,
                                            int rot, int interleaved, int lane_lo, int lane_step) {
  for (int i = lane_lo; i < rot / 2; i += lane_step) {
    const float c = cos[pos * half + i], s = sin[pos * half + i];
    const int i0 = interleaved ? 2 * i : i, i1 = interleaved ? 2 * i + 1 : i + rot / 2;
    const float x0 = v[i0], x1 = v[i1];
    v[i0] = x0 * c - x1 * s;
    v[i1] = x1 * c + x0 * s;
  }
}

// RotaryEmbedding of [B][S] rows of heads x D floats, one warp per (token,
// head): the head is staged in shared memory, rotated in place, written out.
// A position outside [0, max_pos) sets the device error word and passes the
// head through unrotated.
__global__ void __launch_bounds__(256) rotary_kernel(const float *__restrict__ x, int64_t x_rs,
                                                     const int64_t *__restrict__ pos, int pos_per_batch,
                                                     const float *cos, const float *sin, int half, int max_pos,
                                                     float *y, int64_t y_rs, int B, int S, int heads, int D, int rot,
                                                     int interleaved, int32_t *err) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * 8 + warp;
  if (item >= (int64_t)B * S * heads) return;
  const int h = (int)(item % heads);
  const int64_t bs = item / heads;
  const int s = (int)(bs % S), b = (int)(bs / S);
  const int64_t p = pos[(pos_per_batch ? (int64_t)b * S : 0) + s];
  __shared__ float hb[8][256];
  float *v = hb[warp];
  const float *src = x + bs * x_rs + (int64_t)h * D;
  for (int d = lane; d < D; d += 32) v[d] = src[d];
  __syncwarp();
  if (p >= 0 && p < max_pos) {
    rotate_head(v, cos, sin, p, half, rot, interleaved, lane, 32);
  } else if (lane == 0 && err) {
    b2m::set_dev_error(err, B2M_DEVERR_INDEX);
  }
  __syncwarp();
  float *dst = y + bs * y_rs + (int64_t)h * D;
  for (int d = lane; d < D; d += 32) dst[d] = v[d];
}

struct GqaArgs {
  const float *q, *k, *v;   // [B][S][H*D], [B][S][KVH*D] (row strides below)
  int64_t q_rs, kv_rs;      // floats between consecutive tokens
  float *kcache, *vcache;   // [B][KVH][CAP][D]
  const int32_t *past;      // [B] positions already cached (device memory)
  const float *cos, *sin;   // [max_pos][half] or null (no rotary)
  int half, rot, interleaved;
  float *out;               // [B][S][H*D]
  int B, S, H, KVH, D, CAP;
  float scale;
  int32_t *err;
  // Key / value addressing for the attend kernels: element (b, kvh, key j, d)
  // sits at kcache[b*kc_bs + kvh*kc_hs + j*kc_rs + d] (same for vcache). The
  // cache layout gives (KVH*CAP*D, CAP*D, D); MultiHeadAttention reads the
  // projected [B][T][KVH*D] rows directly.
  int64_t kc_bs, kc_hs, kc_rs;
  int causal;               // 1: query i sees keys [0, past + i]; 0: keys [0, kv_len)
  int kv_len;
  // Additive score bias or null: element (b, query head h, query s, key j)
  // at mask[b*mask_bs + h*mask_hs + s*mask_qs + j] (0 strides broadcast).
  const float *mask;
  int64_t mask_bs, mask_hs, mask_qs;
  // Optional f16 copy of `out` (round to nearest), the operand of the output
  // projection's tensor-core GEMM, and optional bf16 hi / lo planes of `out`
  // (row stride H*D), the A operand of a FAST fp32 Gemm.
  __half *out16 = nullptr;
  __nv_bfloat16 *p0 = nullptr, *p1 = nullptr;
  // Decode kernel only: per-head RMSNorm gains of q and k ([H + KVH][D]: the
  // query heads' rows, then the kv heads'), or null when q and k arrive
  // normalised; with them the kernel also appends the token's key and value.
  const float *qk_gain = nullptr;
  double qk_eps = 0.0;
};

// RMSNorm of one head of D <= 128 values held as one float4 per lane (lanes
// at or past D / 4 hold zeros), gain row g: the arithmetic of
// norm_warp4_kernel<1, false> (and of norm_row_cta_kernel with one warp), so
// the result equals the head-rows norm launch bit for bit.
__device__ __forceinline__ float4 rms_head4(float4 v, const float *__restrict__ g, int D, double eps, int lane) {
  const int d4 = D >> 2;
  const float mean = 0.f;
  float s2 = 0.f;
  if (lane < d4) {
    const float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
    s2 = fmaf(a, a, fmaf(b, b, fmaf(c, c, fmaf(d, d, s2))));
  }
  const float inv = (float)(1.0 / sqrt((double)warp_sum_f(s2) / D + eps));
  if (lane >= d4) return make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 gg = reinterpret_cast<const float4 *>(g)[lane];
  const float bb = 0.f;
  return make_float4((v.x - mean) * inv * gg.x + bb, (v.y - mean) * inv * gg.y + bb, (v.z - mean) * inv * gg.z + bb,
                     (v.w - mean) * inv * gg.w + bb);
}

// Sum of squares of a row of D = 64 or 128 values held as one float4 per
// lane by D / 4 consecutive lanes (two rows per warp at D = 64), as
// rms_head4 forms it; every lane of the row gets the sum. At D = 64 the
// butterfly skips the step that would add the other half's zeros in
// rms_head4, which changes no bit.
template <int D>
__device__ __forceinline__ float row_sumsq4(float4 v) {
  static_assert(D == 64 || D == 128, "rows of 16 or 32 lanes");
  const float mean = 0.f;
  const float a = v.x - mean, b = v.y - mean, cc = v.z - mean, d = v.w - mean;
  float t = fmaf(a, a, fmaf(b, b, fmaf(cc, cc, fmaf(d, d, 0.f))));
  if (D == 128) t += __shfl_xor_sync(0xffffffffu, t, 16);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// rms_head4's output arithmetic for float4 c of a row with factor inv.
__device__ __forceinline__ float4 rms_scale4(float4 v, float inv, const float *__restrict__ g, int c) {
  const float mean = 0.f, bb = 0.f;
  const float4 gg = reinterpret_cast<const float4 *>(g)[c];
  return make_float4((v.x - mean) * inv * gg.x + bb, (v.y - mean) * inv * gg.y + bb, (v.z - mean) * inv * gg.z + bb,
                     (v.w - mean) * inv * gg.w + bb);
}

// Appends this call's keys / values to the cache (rotary on K), one warp per
// (token, kv head). With a.qk_gain (D <= 128, float4-aligned rows) each key
// head is RMS-normalised first.
__global__ void __launch_bounds__(256) gqa_append_kernel(const GqaArgs a) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * 8 + warp;
  const int64_t total = (int64_t)a.B * a.S * a.KVH;
  if (item >= total) return;
  const int kvh = (int)(item % a.KVH);
  const int64_t bs = item / a.KVH;
  const int s = (int)(bs % a.S), b = (int)(bs / a.S);
  const int past = a.past[b];
  const int pos = past + s;
  if (pos >= a.CAP) {
    if (lane == 0 && a.err) b2m::set_dev_error(a.err, B2M_DEVERR_CACHE_FULL);
    return;
  }
  __shared__ __align__(16) float kbuf[8][256];
  float *kv = kbuf[warp];
  const float *ksrc = a.k + (int64_t)(b * a.S + s) * a.kv_rs + kvh * a.D;
  const float *vsrc = a.v + (int64_t)(b * a.S + s) * a.kv_rs + kvh * a.D;
  const int64_t dst = (((int64_t)b * a.KVH + kvh) * a.CAP + pos) * a.D;
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const int d4 = a.D >> 2;
  if ((a.D & 3) == 0 && (a.kv_rs & 3) == 0 && al(a.k) && al(a.v) && al(a.kcache) && al(a.vcache)) {
    // float4 rows (D <= 256: at most two per lane); V's loads go out first.
    float4 vv[2];
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (lane + 32 * i < d4) vv[i] = reinterpret_cast<const float4 *>(vsrc)[lane + 32 * i];
    if (a.qk_gain) {
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (lane < d4) x = *reinterpret_cast<const float4 *>(ksrc + 4 * lane);
      const float4 o = rms_head4(x, a.qk_gain + (int64_t)(a.H + kvh) * a.D, a.D, a.qk_eps, lane);
      if (lane < d4) *reinterpret_cast<float4 *>(kv + 4 * lane) = o;
    } else {
#pragma unroll
      for (int i = 0; i < 2; i++)
        if (lane + 32 * i < d4)
          reinterpret_cast<float4 *>(kv)[lane + 32 * i] = reinterpret_cast<const float4 *>(ksrc)[lane + 32 * i];
    }
    __syncwarp();
    if (a.cos) rotate_head(kv, a.cos, a.sin, pos, a.half, a.rot, a.interleaved, lane, 32);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (lane + 32 * i < d4) {
        reinterpret_cast<float4 *>(a.kcache + dst)[lane + 32 * i] = reinterpret_cast<const float4 *>(kv)[lane + 32 * i];
        reinterpret_cast<float4 *>(a.vcache + dst)[lane + 32 * i] = vv[i];
      }
    return;
  }
  for (int d = lane; d < a.D; d += 32) kv[d] = ksrc[d];  // (qk_gain is only set on the float4 layout)
  __syncwarp();
  if (a.cos) rotate_head(kv, a.cos, a.sin, pos, a.half, a.rot, a.interleaved, lane, 32);
  __syncwarp();
  for (int d = lane; d < a.D; d += 32) {
    a.kcache[dst + d] = kv[d];
    a.vcache[dst + d] = vsrc[d];
  }
}

// Causal attention of a tile of query tokens of one (batch, query head)
// against the cache [0, past + s]. One warp per query token: q (rotated) in
// registers across lanes, online softmax over the keys, fp32 accumulation of
// P.V in registers (D <= 256, 8 values per lane).
__global__ void __launch_bounds__(256) gqa_attend_kernel(const GqaArgs a) {
  b2m::pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int s = blockIdx.x * 8 + warp;
  if (s >= a.S) return;
  const int kvh = h / (a.H / a.KVH);
  const int past = a.past ? a.past[b] : 0;
  const int pos = past + s;
  __shared__ float qbuf[8][256];
  float *qv = qbuf[warp];
  const float *qsrc = a.q + (int64_t)(b * a.S + s) * a.q_rs + h * a.D;
  for (int d = lane; d < a.D; d += 32) qv[d] = qsrc[d];
  __syncwarp();
  if (a.cos) rotate_head(qv, a.cos, a.sin, pos, a.half, a.rot, a.interleaved, lane, 32);
  __syncwarp();
  float qr[8];
#pragma unroll
  for (int i = 0; i < 8; i++) qr[i] = lane + 32 * i < a.D ? qv[lane + 32 * i] : 0.f;
  const float *kc = a.kcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  const float *vc = a.vcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  const float *mk = a.mask ? a.mask + (int64_t)b * a.mask_bs + (int64_t)h * a.mask_hs + (int64_t)s * a.mask_qs
                           : nullptr;
  float m = -INFINITY, l = 0.f;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i] = 0.f;
  const int last = a.causal ? (pos < a.CAP ? pos : a.CAP - 1) : a.kv_len - 1;
  for (int j = 0; j <= last; j++) {
    const float *kr = kc + (int64_t)j * a.kc_rs;
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (lane + 32 * i < a.D) part = fmaf(qr[i], kr[lane + 32 * i], part);
    float sc = warp_sum_f(part) * a.scale;
    if (mk) sc += mk[j];
    const float mn = fmaxf(m, sc);
    if (mn == -INFINITY) continue;  // every key so far masked out
    const float corr = __expf(m - mn), p = __expf(sc - mn);
    l = l * corr + p;
    const float *vr = vc + (int64_t)j * a.kc_rs;
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (lane + 32 * i < a.D) acc[i] = fmaf(p, vr[lane + 32 * i], acc[i] * corr);
    m = mn;
  }
  float *dst = a.out + (int64_t)(b * a.S + s) * (int64_t)a.H * a.D + h * a.D;
  const float inv = 1.f / l;
#pragma unroll
  for (int i = 0; i < 8; i++)
    if (lane + 32 * i < a.D) dst[lane + 32 * i] = acc[i] * inv;
}

// Flash-style attention for multi-token calls (prefill), fp32 on the CUDA
// cores. CTA = (64-query tile, query head, batch), 256 threads. Each thread
// owns 4 query rows x 4 keys of the 64 x 64 score tile and the same 4 rows x
// D/16 columns of the output; the row statistics of the online softmax
// (max, sum) are reduced over the 16 threads that share the rows. Q is
// rotated and pre-scaled on load; K (rotated by gqa_append_kernel) and V come
// from the cache. Key tiles past the last visible key are skipped.
template <int D>
__global__ void __launch_bounds__(256) gqa_prefill_kernel(const GqaArgs a) {
  b2m::pdl_launch_dependents();
  constexpr int QT = 64, KT = 64, LD = 68, CPT = D / 16;
  extern __shared__ __align__(16) float fsm[];
  float *Qt = fsm;            // [D][LD], Qt[d][r]
  float *Kt = Qt + D * LD;    // [D][LD], Kt[d][c]
  float *Vs = Kt + D * LD;    // [KT][D]
  float *Ps = Vs + KT * D;    // [QT][LD]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int h = blockIdx.y, b = blockIdx.z, q0 = blockIdx.x * QT;
  const int kvh = h / (a.H / a.KVH);
  const int past = a.past ? a.past[b] : 0;
  for (int i = tid; i < QT * D; i += 256) {
    const int r = i / D, d = i % D;
    const int s = q0 + r;
    Qt[d * LD + r] = s < a.S ? a.q[(int64_t)(b * a.S + s) * a.q_rs + h * D + d] * a.scale : 0.f;
  }
  __syncthreads();
  if (a.cos) {
    const int npair = a.rot / 2;
    for (int i = tid; i < QT * npair; i += 256) {
      const int r = i / npair, pi = i % npair;
      const int64_t pos = past + q0 + r;
      if (q0 + r >= a.S || pos >= a.CAP) continue;
      const float c = a.cos[pos * a.half + pi], sn = a.sin[pos * a.half + pi];
      const int i0 = a.interleaved ? 2 * pi : pi, i1 = a.interleaved ? 2 * pi + 1 : pi + npair;
      const float x0 = Qt[i0 * LD + r], x1 = Qt[i1 * LD + r];
      Qt[i0 * LD + r] = x0 * c - x1 * sn;
      Qt[i1 * LD + r] = x1 * c + x0 * sn;
    }
  }
  const int last_q = min(q0 + QT, a.S) - 1;
  const int max_key = a.causal ? min(past + last_q, a.CAP - 1) : a.kv_len - 1;
  const float *kc = a.kcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  const float *vc = a.vcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  const float *mk = a.mask ? a.mask + (int64_t)b * a.mask_bs + (int64_t)h * a.mask_hs : nullptr;
  const bool per_query = mk && a.mask_qs != 0;  // else one bias row shared by all queries
  __shared__ float mrow[64];
  float m[4], l[4], o[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < CPT; c++) o[i][c] = 0.f;
  }
  for (int j0 = 0; j0 <= max_key; j0 += KT) {
    __syncthreads();
    for (int i = tid; i < KT * D; i += 256) {
      const int c = i / D, d = i % D;
      const int j = j0 + c;
      const bool ok = j <= max_key;
      Kt[d * LD + c] = ok ? kc[(int64_t)j * a.kc_rs + d] : 0.f;
      Vs[c * D + d] = ok ? vc[(int64_t)j * a.kc_rs + d] : 0.f;
    }
    if (tid < KT) {
      const int j = j0 + tid;
      mrow[tid] = j > max_key ? -INFINITY : (mk && !per_query ? mk[j] : 0.f);
    }
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; d++) {
      const float4 qv = *reinterpret_cast<const float4 *>(&Qt[d * LD + ty * 4]);
      const float4 kv = *reinterpret_cast<const float4 *>(&Kt[d * LD + tx * 4]);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) sc[i][j] = fmaf(qa[i], ka[j], sc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int qpos = past + q0 + ty * 4 + i;
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        sc[i][j] += mrow[tx * 4 + j];
        if (per_query && q0 + ty * 4 + i < a.S && j0 + tx * 4 + j <= max_key)
          sc[i][j] += mk[(int64_t)(q0 + ty * 4 + i) * a.mask_qs + j0 + tx * 4 + j];
        if (a.causal && j0 + tx * 4 + j > qpos) sc[i][j] = -INFINITY;
        rmax = fmaxf(rmax, sc[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      const float mn = fmaxf(m[i], rmax);
      const float corr = mn == -INFINITY ? 1.f : __expf(m[i] - mn);
      float rsum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float pv = mn == -INFINITY ? 0.f : __expf(sc[i][j] - mn);
        Ps[(ty * 4 + i) * LD + tx * 4 + j] = pv;
        rsum += pv;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, off);
      l[i] = l[i] * corr + rsum;
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < CPT; c++) o[i][c] *= corr;
    }
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < KT; j++) {
      float pj[4];
#pragma unroll
      for (int i = 0; i < 4; i++) pj[i] = Ps[(ty * 4 + i) * LD + j];
      const float *vr = Vs + j * D + tx * CPT;
#pragma unroll
      for (int c = 0; c < CPT; c++) {
        const float vv = vr[c];
#pragma unroll
        for (int i = 0; i < 4; i++) o[i][c] = fmaf(pj[i], vv, o[i][c]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int s = q0 + ty * 4 + i;
    if (s >= a.S) continue;
    float *dst = a.out + (int64_t)(b * a.S + s) * (int64_t)a.H * D + h * D + tx * CPT;
    const float inv = 1.f / l[i];
#pragma unroll
    for (int c = 0; c < CPT; c++) dst[c] = o[i][c] * inv;
  }
}

// Sums eight values over the warp and leaves all eight totals in every lane:
// three reduce-scatter rounds (4 + 2 + 1 shuffles) leave value k summed over
// lanes differing in bits 4..2 in lanes whose bits 4..2 spell k, two rounds
// finish the sum, eight shuffles broadcast. 17 shuffles instead of 40.
__device__ __forceinline__ void warp_allreduce8(float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  float t4[4], t2[2];
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float send = h16 ? v[i] : v[i + 4], keep = h16 ? v[i + 4] : v[i];
    t4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const float send = h8 ? t4[i] : t4[i + 2], keep = h8 ? t4[i + 2] : t4[i];
    t2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float t1;
  {
    const float send = h4 ? t2[0] : t2[1], keep = h4 ? t2[1] : t2[0];
    t1 = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  t1 += __shfl_xor_sync(0xffffffffu, t1, 2);
  t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
#pragma unroll
  for (int k = 0; k < 8; k++) v[k] = __shfl_sync(0xffffffffu, t1, k << 2);
}

// Single-token attention (decode): CTA = (kv head, sequence, key split),
// 256 threads, the G query heads of the group together so each cached K/V
// row is read once. A warp takes 8/G keys per step: every lane loads its
// D/32 values of each K and V row (512-byte coalesced rows for D = 128, all
// the step's loads in flight together), the 8 partial dot products are
// reduced together, and the warp's online-softmax state is updated. The 8
// warp states merge in shared memory in fixed order; with key splits the
// split states go to pm / pl / po and gqa_decode_combine_kernel merges them.
template <int D, int G>
__global__ void __launch_bounds__(256) gqa_decode_kernel(const GqaArgs a, float *pm, float *pl, float *po,
                                                         uint32_t *counters) {
  b2m::pdl_launch_dependents();
  constexpr int VPD = D / 32, KB = 8 / G;
  static_assert(D % 32 == 0 && D <= 128 && KB * G == 8, "decode kernel shape");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x, b = blockIdx.y, sp = blockIdx.z, nsplit = gridDim.z;
  const int past = a.past[b];
  const int nkeys = min(past + 1, a.CAP);
  const int chunk = (nkeys + nsplit - 1) / nsplit;
  const int jbeg = sp * chunk, jend = min(nkeys, jbeg + chunk);
  __shared__ __align__(16) float qs[G][D];
  __shared__ float wm[8][G], wl[8][G];
  __shared__ float wo[8][G][D];
  if (a.qk_gain) {
    // Head RMSNorm folded in: warp g normalises query head kvh*G + g; warp
    // G % 8 normalises this kv head's new key, rotates it and appends it and
    // the value at position past, in the CTA whose key range holds past (it
    // reads them back below; __syncthreads makes the stores visible).
    constexpr int D4 = D / 4;
    if (warp < G) {
      const int h = kvh * G + warp;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (lane < D4) x = *reinterpret_cast<const float4 *>(a.q + (int64_t)b * a.q_rs + (int64_t)h * D + 4 * lane);
      const float4 o = rms_head4(x, a.qk_gain + (int64_t)h * D, D, a.qk_eps, lane);
      if (lane < D4) {
        qs[warp][4 * lane + 0] = o.x * a.scale;
        qs[warp][4 * lane + 1] = o.y * a.scale;
        qs[warp][4 * lane + 2] = o.z * a.scale;
        qs[warp][4 * lane + 3] = o.w * a.scale;
      }
    }
    if (warp == (G & 7)) {
      __shared__ __align__(16) float kb[D];
      if (past >= a.CAP) {
        if (lane == 0 && sp == 0 && a.err) b2m::set_dev_error(a.err, B2M_DEVERR_CACHE_FULL);
      } else if (jbeg <= past && past < jend) {
        const float *ksrc = a.k + (int64_t)b * a.kv_rs + (int64_t)kvh * D;
        const float *vsrc = a.v + (int64_t)b * a.kv_rs + (int64_t)kvh * D;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane < D4) x = *reinterpret_cast<const float4 *>(ksrc + 4 * lane);
        const float4 o = rms_head4(x, a.qk_gain + (int64_t)(a.H + kvh) * D, D, a.qk_eps, lane);
        if (lane < D4) *reinterpret_cast<float4 *>(&kb[4 * lane]) = o;
        __syncwarp();
        if (a.cos) rotate_head(kb, a.cos, a.sin, past, a.half, a.rot, a.interleaved, lane, 32);
        __syncwarp();
        const int64_t dst = (((int64_t)b * a.KVH + kvh) * a.CAP + past) * D;
        for (int d = lane; d < D; d += 32) {
          a.kcache[dst + d] = kb[d];
          a.vcache[dst + d] = vsrc[d];
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < G * D; i += 256) {
      const int g = i / D, d = i % D;
      qs[g][d] = a.q[(int64_t)b * a.q_rs + (kvh * G + g) * D + d] * a.scale;
    }
  }
  __syncthreads();
  if (a.cos && past < a.CAP) {
    const int npair = a.rot / 2;
    for (int i = threadIdx.x; i < G * npair; i += 256) {
      const int g = i / npair, pi = i % npair;
      const float c = a.cos[(int64_t)past * a.half + pi], sn = a.sin[(int64_t)past * a.half + pi];
      const int i0 = a.interleaved ? 2 * pi : pi, i1 = a.interleaved ? 2 * pi + 1 : pi + npair;
      const float x0 = qs[g][i0], x1 = qs[g][i1];
      qs[g][i0] = x0 * c - x1 * sn;
      qs[g][i1] = x1 * c + x0 * sn;
    }
  }
  __syncthreads();
  float q[G][VPD];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int c = 0; c < VPD; c++) q[g][c] = qs[g][lane * VPD + c];
  const float *kc = a.kcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs + lane * VPD;
  const float *vc = a.vcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs + lane * VPD;
  float m[G], l[G], o[G][VPD];
#pragma unroll
  for (int g = 0; g < G; g++) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int c = 0; c < VPD; c++) o[g][c] = 0.f;
  }
  // The next step's K / V rows are requested before this step's arithmetic,
  // so a warp always has two steps of loads in flight.
  float kn[KB][VPD], vn[KB][VPD];
  auto load_step = [&](int j0) {
#pragma unroll
    for (int kb = 0; kb < KB; kb++) {
      const bool ok = j0 + kb < jend;
      const float *kp = kc + (int64_t)(j0 + kb) * a.kc_rs, *vp = vc + (int64_t)(j0 + kb) * a.kc_rs;
      if constexpr (VPD == 4) {
        const float4 k4 = ok ? *reinterpret_cast<const float4 *>(kp) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 v4 = ok ? *reinterpret_cast<const float4 *>(vp) : make_float4(0.f, 0.f, 0.f, 0.f);
        kn[kb][0] = k4.x, kn[kb][1] = k4.y, kn[kb][2] = k4.z, kn[kb][3] = k4.w;
        vn[kb][0] = v4.x, vn[kb][1] = v4.y, vn[kb][2] = v4.z, vn[kb][3] = v4.w;
      } else {
#pragma unroll
        for (int c = 0; c < VPD; c++) {
          kn[kb][c] = ok ? kp[c] : 0.f;
          vn[kb][c] = ok ? vp[c] : 0.f;
        }
      }
    }
  };
  if (jbeg + warp * KB < jend) load_step(jbeg + warp * KB);
  for (int j0 = jbeg + warp * KB; j0 < jend; j0 += 8 * KB) {
    float kr[KB][VPD], vr[KB][VPD];
#pragma unroll
    for (int kb = 0; kb < KB; kb++)
#pragma unroll
      for (int c = 0; c < VPD; c++) {
        kr[kb][c] = kn[kb][c];
        vr[kb][c] = vn[kb][c];
      }
    if (j0 + 8 * KB < jend) load_step(j0 + 8 * KB);
    float s[8];
#pragma unroll
    for (int kb = 0; kb < KB; kb++)
#pragma unroll
      for (int g = 0; g < G; g++) {
        float t = 0.f;
#pragma unroll
        for (int c = 0; c < VPD; c++) t = fmaf(q[g][c], kr[kb][c], t);
        s[kb * G + g] = t;
      }
    warp_allreduce8(s);
#pragma unroll
    for (int g = 0; g < G; g++) {
      float mx = m[g];
#pragma unroll
      for (int kb = 0; kb < KB; kb++)
        if (j0 + kb < jend) mx = fmaxf(mx, s[kb * G + g]);
      const float corr = __expf(m[g] - mx);
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < VPD; c++) o[g][c] *= corr;
#pragma unroll
      for (int kb = 0; kb < KB; kb++) {
        const float p = j0 + kb < jend ? __expf(s[kb * G + g] - mx) : 0.f;
        psum += p;
#pragma unroll
        for (int c = 0; c < VPD; c++) o[g][c] = fmaf(p, vr[kb][c], o[g][c]);
      }
      l[g] = l[g] * corr + psum;
      m[g] = mx;
    }
  }
#pragma unroll
  for (int g = 0; g < G; g++) {
    if (lane == 0) {
      wm[warp][g] = m[g];
      wl[warp][g] = l[g];
    }
#pragma unroll
    for (int c = 0; c < VPD; c++) wo[warp][g][lane * VPD + c] = o[g][c];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += 256) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < 8; w++) M = fmaxf(M, wm[w][g]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 8; w++) {
      const float f = wm[w][g] == -INFINITY ? 0.f : __expf(wm[w][g] - M);
      L += wl[w][g] * f;
      O += wo[w][g][d] * f;
    }
    const int h = kvh * G + g;
    if (nsplit == 1) {
      const float ov = O / L;
      if (a.out) a.out[(int64_t)b * (int64_t)a.H * D + h * D + d] = ov;
      if (a.out16) a.out16[(int64_t)b * (int64_t)a.H * D + h * D + d] = __float2half_rn(ov);
    } else {
      const int64_t slot = ((int64_t)b * a.H + h) * nsplit + sp;
      if (d == 0) {
        pm[slot] = M;
        pl[slot] = L;
      }
      po[slot * D + d] = O;
    }
  }
  if (nsplit > 1 && counters) {
    // The last split CTA of this (kv head, sequence) to finish merges the
    // split states in split order, exactly as gqa_decode_combine_kernel does,
    // and re-arms the counter for the next call (calls are stream-ordered).
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&counters[(int64_t)b * a.KVH + kvh], 1u) == (uint32_t)(nsplit - 1);
    __syncthreads();
    if (last) {
      __threadfence();
      for (int i = threadIdx.x; i < G * D; i += 256) {
        const int g = i / D, d = i % D;
        const int h = kvh * G + g;
        const int64_t base = ((int64_t)b * a.H + h) * nsplit;
        float M = -INFINITY;
        for (int s2 = 0; s2 < nsplit; s2++) M = fmaxf(M, __ldcg(pm + base + s2));
        float L = 0.f, O = 0.f;
        for (int s2 = 0; s2 < nsplit; s2++) {
          const float mv = __ldcg(pm + base + s2);
          const float f = mv == -INFINITY ? 0.f : __expf(mv - M);
          L += __ldcg(pl + base + s2) * f;
          O += __ldcg(po + (base + s2) * D + d) * f;
        }
          const float ov = O / L;
        if (a.out) a.out[(int64_t)b * (int64_t)a.H * D + h * D + d] = ov;
        if (a.out16) a.out16[(int64_t)b * (int64_t)a.H * D + h * D + d] = __float2half_rn(ov);
      }
      if (threadIdx.x == 0) counters[(int64_t)b * a.KVH + kvh] = 0u;
    }
  }
}

// Merges the key-split states of gqa_decode_kernel in split order.
__global__ void gqa_decode_combine_kernel(const float *pm, const float *pl, const float *po, float *out, int H, int D,
                                          int nsplit) {
  b2m::pdl_launch_dependents();
  const int h = blockIdx.x, b = blockIdx.y;
  const int64_t base = ((int64_t)b * H + h) * nsplit;
  float M = -INFINITY;
  for (int sp = 0; sp < nsplit; sp++) M = fmaxf(M, pm[base + sp]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int sp = 0; sp < nsplit; sp++) {
      const float f = pm[base + sp] == -INFINITY ? 0.f : __expf(pm[base + sp] - M);
      L += pl[base + sp] * f;
      O += po[(base + sp) * D + d] * f;
    }
    out[((int64_t)b * H + h) * D + d] = O / L;
  }
}

// ---------------------------------------------------------------------------
// MultiHeadAttention on the tensor cores for one (query head, sequence) of at
// most 128 queries x 128 keys, head_dim 64 (the BERT-base shape). Scores and
// P.V are fp32 products of bf16-split operands (x = x0 + x1, three
// kind::f16 MMAs per product, ~1e-5 relative), the softmax runs in fp32 on
// the accumulator rows.
//
//   smem (bytes, 128-byte-swizzled K-major [rows][64 bf16] blocks):
//     [0, 64K)    Q hi, Q lo, K hi, K lo (16 KB each); later P hi / lo
//                 ([128 queries][128 keys], two 64-key blocks each), later
//                 the output staging
//     [64K, 96K)  V^T hi, V^T lo: [64 dims][128 keys], two 64-key blocks
//     [96K, ...)  bias row (128 floats), barriers, TMEM slot
//   TMEM: scores in columns [0, 128), output in [128, 192).
// ---------------------------------------------------------------------------
using b2m::fence_proxy_async_smem;
using b2m::mbar_fence_init;
using b2m::mbar_init;
using b2m::smem_u32;
using b2m::split_bf16x2;
using b2m::sw128_kmajor_desc;
using b2m::tc_fence_after;
using b2m::tc_fence_before;
using b2m::tmem_alloc;
using b2m::tmem_dealloc;
using b2m::tmem_ld16;
using b2m::tmem_ld_wait;
using b2m::tmem_st8;
using b2m::tmem_st_wait;
using b2m::umma_commit;
using b2m::umma_f16;
using b2m::umma_f16_ts;
using b2m::umma_idesc;
using b2m::warp_wait_or_abort;

constexpr int MTC_D = 64;
constexpr uint32_t MTC_QH = 0, MTC_QL = 16384, MTC_KH = 32768, MTC_KL = 49152;
constexpr uint32_t MTC_PH = 0, MTC_PL = 32768;
constexpr uint32_t MTC_VH = 65536, MTC_VL = 81920;
constexpr uint32_t MTC_MASK = 98304, MTC_BAR = MTC_MASK + 512, MTC_SLOT = MTC_BAR + 16;
constexpr uint32_t MTC_BYTES = MTC_SLOT + 16 + 1024;

// Byte offset of bf16 element (row r, k) in a [rows][64] SW128 K-major block.
__device__ __forceinline__ uint32_t sw128_elem(int r, int k) {
  return (uint32_t)(r * 128 + ((((k >> 3) ^ (r & 7)) << 4) | ((k & 7) << 1)));
}

// x = x0 + x1 in bf16 (x0 = rn(x), truncated if rounding would overflow a
// finite x; x1 = rn(x - x0), 0 for non-finite x).
__device__ __forceinline__ void split2_bf16(float x, __nv_bfloat16 &h, __nv_bfloat16 &l) {
  h = __float2bfloat16_rn(x);
  float hf = __bfloat162float(h);
  if (isinf(hf) && isfinite(x)) {
    h = __float2bfloat16_rz(x);
    hf = __bfloat162float(h);
  }
  l = __float2bfloat16_rn(isfinite(x) ? x - hf : 0.f);
}

// Stages one [128][64] fp32 operand (row r of 64 floats at base + r * rs,
// rows >= n are zero) as bf16 hi / lo SW128 blocks. Item (row, 8-float
// chunk), 1024 per operand over the CTA's threads: a warp reads four 256-byte
// row segments.
__device__ __forceinline__ void mtc_stage_rows(uint8_t *smem, uint32_t off_h, uint32_t off_l, const float *base,
                                               int64_t rs, int n) {
  for (int it = threadIdx.x; it < 128 * 8; it += blockDim.x) {
    const int r = it >> 3, c = it & 7;
    float x[8];
    if (r < n) {
      const float *src = base + (int64_t)r * rs + 8 * c;
      const float4 a = *reinterpret_cast<const float4 *>(src);
      const float4 b = *reinterpret_cast<const float4 *>(src + 4);
      x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) x[j] = 0.f;
    }
    __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; j++) split2_bf16(x[j], h[j], l[j]);
    *reinterpret_cast<uint4 *>(smem + off_h + sw128_elem(r, 8 * c)) = *reinterpret_cast<const uint4 *>(h);
    *reinterpret_cast<uint4 *>(smem + off_l + sw128_elem(r, 8 * c)) = *reinterpret_cast<const uint4 *>(l);
  }
}

// 512 threads. Warp w reads TMEM lane quarter w % 4 (query rows) and owns
// column block w / 4: 32 of the 128 score columns, 16 of the 64 output
// columns; row max and sum combine the four column blocks in shared memory.
__global__ void __launch_bounds__(512) mha_tc_kernel(const GqaArgs a) {
  b2m::pdl_launch_dependents();
  extern __shared__ uint8_t mtc_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(mtc_raw) + 1023) & ~(uintptr_t)1023);
  float *mrow = reinterpret_cast<float *>(smem + MTC_MASK);
  uint64_t *bar_s = reinterpret_cast<uint64_t *>(smem + MTC_BAR), *bar_o = bar_s + 1;
  uint32_t *slot = reinterpret_cast<uint32_t *>(smem + MTC_SLOT);
  __shared__ int abort_flag_s;
  __shared__ float red[4][128];
  volatile int *abort_flag = &abort_flag_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int q4 = warp & 3, cb = warp >> 2;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kvh = h / (a.H / a.KVH);
  const int S = a.S, T = a.kv_len;
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    abort_flag_s = 0;
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(slot, 256);
  mtc_stage_rows(smem, MTC_QH, MTC_QL, a.q + (int64_t)b * S * a.q_rs + h * MTC_D, a.q_rs, S);
  const float *kb0 = a.kcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  const float *vb0 = a.vcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  mtc_stage_rows(smem, MTC_KH, MTC_KL, kb0, a.kc_rs, T);
  {
    // V^T: thread packs keys 2p, 2p+1 of dims 8g .. 8g+7 as bf16 pairs.
    const int pr = tid & 63, g = tid >> 6;
    const int t0 = 2 * pr;
    const float *v0 = vb0 + (int64_t)t0 * a.kc_rs + 8 * g, *v1 = v0 + a.kc_rs;
    float e0[8], e1[8];
#pragma unroll
    for (int j = 0; j < 8; j++) e0[j] = e1[j] = 0.f;
    if (t0 < T) {
      const float4 x = *reinterpret_cast<const float4 *>(v0), y = *reinterpret_cast<const float4 *>(v0 + 4);
      e0[0] = x.x, e0[1] = x.y, e0[2] = x.z, e0[3] = x.w, e0[4] = y.x, e0[5] = y.y, e0[6] = y.z, e0[7] = y.w;
    }
    if (t0 + 1 < T) {
      const float4 x = *reinterpret_cast<const float4 *>(v1), y = *reinterpret_cast<const float4 *>(v1 + 4);
      e1[0] = x.x, e1[1] = x.y, e1[2] = x.z, e1[3] = x.w, e1[4] = y.x, e1[5] = y.y, e1[6] = y.z, e1[7] = y.w;
    }
    const uint32_t blk = (uint32_t)(t0 >> 6) * 8192u;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      __nv_bfloat16 h0, l0, h1, l1;
      split2_bf16(e0[j], h0, l0);
      split2_bf16(e1[j], h1, l1);
      const uint32_t o = blk + sw128_elem(8 * g + j, t0 & 63);
      *reinterpret_cast<__nv_bfloat162 *>(smem + MTC_VH + o) = __halves2bfloat162(h0, h1);
      *reinterpret_cast<__nv_bfloat162 *>(smem + MTC_VL + o) = __halves2bfloat162(l0, l1);
    }
  }
  const float *mk = a.mask ? a.mask + (int64_t)b * a.mask_bs + (int64_t)h * a.mask_hs : nullptr;
  const bool per_query = mk && a.mask_qs != 0;
  if (tid < 128) mrow[tid] = tid >= T ? -INFINITY : (mk && !per_query ? mk[tid] : 0.f);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (tid == 0) {
    constexpr uint32_t idesc_s = umma_idesc(128, 128, 1u, 1u, 1u);
    const uint32_t base = smem_u32(smem);
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const uint32_t o = (uint32_t)kk * 32u;
      const uint64_t qh = sw128_kmajor_desc(base + MTC_QH + o), ql = sw128_kmajor_desc(base + MTC_QL + o);
      const uint64_t kh = sw128_kmajor_desc(base + MTC_KH + o), kl = sw128_kmajor_desc(base + MTC_KL + o);
      umma_f16(tmem, ql, kh, idesc_s, kk ? 1u : 0u);
      umma_f16(tmem, qh, kl, idesc_s, 1u);
      umma_f16(tmem, qh, kh, idesc_s, 1u);
    }
    umma_commit(bar_s);
  }
  const bool ok_s = warp_wait_or_abort(bar_s, 0u, abort_flag, a.err);
  tc_fence_after();
  // Softmax of query row r over this warp's 32 key columns (fp32); P
  // (unnormalised, <= 1) goes to shared memory as bf16 hi / lo.
  const int r = q4 * 32 + lane, c0 = cb * 32;
  const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
  const float *mq = per_query && r < S ? mk + (int64_t)r * a.mask_qs : nullptr;
  float sv[32];
  float mx = -INFINITY;
  if (ok_s) {
    uint32_t v[32];
    tmem_ld16(trow + (uint32_t)c0, *reinterpret_cast<uint32_t(*)[16]>(v));
    tmem_ld16(trow + (uint32_t)c0 + 16u, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const int t = c0 + j;
      float x = __uint_as_float(v[j]) * a.scale + mrow[t];
      if (mq && t < T) x += mq[t];
      if (a.causal && t > r) x = -INFINITY;
      sv[j] = x;
      mx = fmaxf(mx, x);
    }
  }
  red[cb][r] = mx;
  __syncthreads();  // also: every S read is done before P overwrites Q / K
  mx = fmaxf(fmaxf(red[0][r], red[1][r]), fmaxf(red[2][r], red[3][r]));
  float psum = 0.f;
  if (ok_s) {
    __align__(16) __nv_bfloat16 ph[32], pl[32];
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const float e = mx == -INFINITY ? 0.f : __expf(sv[j] - mx);
      psum += e;
      split2_bf16(e, ph[j], pl[j]);
    }
    const uint32_t blk = (uint32_t)(c0 >> 6) * 16384u;
#pragma unroll
    for (int hh = 0; hh < 4; hh++) {
      const uint32_t o = blk + sw128_elem(r, (c0 & 63) + 8 * hh);
      *reinterpret_cast<uint4 *>(smem + MTC_PH + o) = *reinterpret_cast<const uint4 *>(ph + 8 * hh);
      *reinterpret_cast<uint4 *>(smem + MTC_PL + o) = *reinterpret_cast<const uint4 *>(pl + 8 * hh);
    }
  }
  __syncthreads();  // every thread has read red[][] (max) before it is reused
  red[cb][r] = psum;
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const float lsum = (red[0][r] + red[1][r]) + (red[2][r] + red[3][r]);
  if (tid == 0 && ok_s) {
    constexpr uint32_t idesc_o = umma_idesc(128, 64, 1u, 1u, 1u);
    const uint32_t base = smem_u32(smem);
#pragma unroll
    for (int kk = 0; kk < 8; kk++) {
      const uint32_t o = (uint32_t)(kk & 3) * 32u;
      const uint64_t ph = sw128_kmajor_desc(base + MTC_PH + (kk >> 2) * 16384u + o);
      const uint64_t pl = sw128_kmajor_desc(base + MTC_PL + (kk >> 2) * 16384u + o);
      const uint64_t vh = sw128_kmajor_desc(base + MTC_VH + (kk >> 2) * 8192u + o);
      const uint64_t vl = sw128_kmajor_desc(base + MTC_VL + (kk >> 2) * 8192u + o);
      umma_f16(tmem + 128, pl, vh, idesc_o, kk ? 1u : 0u);
      umma_f16(tmem + 128, ph, vl, idesc_o, 1u);
      umma_f16(tmem + 128, ph, vh, idesc_o, 1u);
    }
  }
  if (tid == 0) umma_commit(bar_o);  // also when skipped, so every wait ends
  const bool ok_o = warp_wait_or_abort(bar_o, 0u, abort_flag, a.err) && ok_s;
  tc_fence_after();
  __syncthreads();  // the MMAs' P reads are complete: the staging may reuse it
  // Output O / l: this warp's 16 columns of its 32 rows into a [128][65]
  // staging block, then row-contiguous stores by all threads.
  float *st = reinterpret_cast<float *>(smem);
  if (ok_o) {
    const float inv = 1.f / lsum;
    uint32_t v[16];
    tmem_ld16(trow + 128u + (uint32_t)(cb * 16), v);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; j++) st[r * 65 + cb * 16 + j] = __uint_as_float(v[j]) * inv;
  }
  __syncthreads();
  if (ok_o) {
    for (int it = tid; it < 128 * MTC_D; it += 512) {
      const int q = it >> 6, d = it & 63;
      if (q < S) {
        const int64_t idx = ((int64_t)b * S + q) * (int64_t)a.H * MTC_D + h * MTC_D + d;
        const float x = st[q * 65 + d];
        a.out[idx] = x;
        if (a.p0) b2m::split_bf16(x, a.p0[idx], a.p1[idx]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// Causal GroupQueryAttention prefill on the tensor cores (head_dim 64 or
// 128, keys from the KV cache): flash-style, one CTA of 512 threads per
// (128-query tile, query head, sequence), 64-key tiles with an online
// softmax. Q (scaled, then rotated as the SIMT prefill kernel does) is split
// into bf16 hi / lo planes once. Per key tile j:
//   * Q.K_j^T, three kind::f16 products (the bf16 split Q0.K0 + Q0.K1 +
//     Q1.K0, as the FAST GEMM) into TMEM columns 0-63, was issued at the end
//     of tile j-1; meanwhile all threads split tile j+1's K and V^T (loaded
//     into registers one tile earlier) into the other of two shared-memory
//     buffers and load tile j+2;
//   * warp w reads lane quarter w % 4 (query rows) and 16 of the 64 score
//     columns, applies the causal limit (key j visible to query i when
//     j <= past + i); the four column warps of a row agree on the running max
//     and sum through shared memory; P = exp(s - max), split into bf16 hi /
//     lo, goes to TMEM with tcgen05.st;
//   * one thread issues P.V with P as the TMEM (A) operand (three products
//     into TMEM columns 64 .. 64 + D) and, behind it, Q.K_{j+1}^T; each thread
//     folds its D / 4 output columns into registers as O = O * corr + PV.
// Every wait is bounded; a timeout records the device error and the CTA
// leaves the loop.
// ---------------------------------------------------------------------------
template <int D>
struct FaLayout {
  static constexpr int ND = D / 64;                       // 64-dim SW128 blocks of Q / K
  static constexpr uint32_t QH = 0, QL = ND * 16384;      // [128][64] blocks
  static constexpr uint32_t R = 2 * ND * 16384;           // K / V buffers (Q staging scratch first)
  // Two K / V buffers, KV_BUF apart: K hi / lo [64][64] blocks, then V^T
  // hi / lo [D][64] blocks.
  static constexpr uint32_t KH = R, KL = KH + ND * 8192;
  static constexpr uint32_t VH = KL + ND * 8192, VL = VH + D * 128;
  static constexpr uint32_t KV_BUF = 2 * ND * 8192 + 2 * D * 128;
  static constexpr uint32_t RED = R + 2 * KV_BUF;         // red_m[4][128], red_l[4][128]
  static constexpr uint32_t BAR = RED + 2 * 4 * 128 * 4;  // bar_s, bar_o
  static constexpr uint32_t SLOT = BAR + 16;
  static constexpr uint32_t FLAG = SLOT + 8;
  static constexpr uint32_t BYTES = FLAG + 8 + 1024;      // + alignment slack
  // TMEM columns: S [0, 64), the P.V accumulator [64, 64 + D), P as bf16
  // hi / lo pairs (32 columns each).
  static constexpr uint32_t P_HI = 64 + D, P_LO = P_HI + 32;
  static_assert(P_LO + 32 <= 256, "TMEM allocation");
  static_assert(128 * D * 4 <= 2 * KV_BUF, "Q staging fits the K / V buffers");
  static_assert(BYTES <= 232448, "shared memory");
};

template <int D>
__global__ void __launch_bounds__(512, 1) fa_tc_kernel(const GqaArgs a) {
  b2m::pdl_launch_dependents();
  using L = FaLayout<D>;
  constexpr int DW = D / 4;  // output columns per thread
  extern __shared__ uint8_t fa_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~(uintptr_t)1023);
  float *red_m = reinterpret_cast<float *>(smem + L::RED), *red_l = red_m + 4 * 128;
  uint64_t *bar_s = reinterpret_cast<uint64_t *>(smem + L::BAR), *bar_o = bar_s + 1;
  uint32_t *slot = reinterpret_cast<uint32_t *>(smem + L::SLOT);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int q4 = warp & 3, cb = warp >> 2;
  const int q0 = blockIdx.x * 128, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.H / a.KVH);
  const int past = a.past[b];
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(slot, 256);

  // Q tile: scaled fp32 rows in the K / V / P region, rotated, then split.
  // Every load of a phase is issued before its first use (the rotary pass
  // read cos / sin one pair at a time and took ~20,000 cycles per CTA).
  float *qf = reinterpret_cast<float *>(smem + L::R);  // [128][D]
  {
    constexpr int QI = 128 * (D / 4) / 512;  // float4 items per thread
    float4 qv[QI];
#pragma unroll
    for (int u = 0; u < QI; u++) {
      const int e = tid + 512 * u, rr = e / (D / 4), c = e % (D / 4);
      qv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q0 + rr < a.S)
        qv[u] = *reinterpret_cast<const float4 *>(a.q + (int64_t)(b * a.S + q0 + rr) * a.q_rs + h * D + 4 * c);
    }
    float inv[QI];
    if (a.qk_gain) {
      // The head's RMSNorm folded in. A warp holds eight rows over its items
      // (one per item at D = 128, two at D = 64, half a warp each); lane l
      // forms the double-precision factor of row l % 8 alone and the factors
      // come back by shuffle: an eighth of the FP64 work of every lane
      // forming every factor, the same bits.
      static_assert(QI * 32 / (D / 4) == 8, "eight rows per warp");
      float ts[QI];
#pragma unroll
      for (int u = 0; u < QI; u++) ts[u] = row_sumsq4<D>(qv[u]);
      const int myrow = lane & 7;
      float mine = 0.f;
#pragma unroll
      for (int u = 0; u < QI; u++) {
        if (D == 128) {
          if (myrow == u) mine = ts[u];
        } else {
          const float t0 = __shfl_sync(0xffffffffu, ts[u], 0), t1 = __shfl_sync(0xffffffffu, ts[u], 16);
          if (myrow == 2 * u) mine = t0;
          if (myrow == 2 * u + 1) mine = t1;
        }
      }
      const float inv_l = (float)(1.0 / sqrt((double)mine / D + a.qk_eps));
#pragma unroll
      for (int u = 0; u < QI; u++) inv[u] = __shfl_sync(0xffffffffu, inv_l, D == 128 ? u : 2 * u + (lane >> 4));
    }
#pragma unroll
    for (int u = 0; u < QI; u++) {
      const int e = tid + 512 * u, rr = e / (D / 4), c = e % (D / 4);
      float4 v = qv[u];
      if (a.qk_gain) {  // padding rows stay zero
        const float4 o = rms_scale4(v, inv[u], a.qk_gain + (int64_t)h * D, c);
        if (q0 + rr < a.S) v = o;
      }
      v.x *= a.scale, v.y *= a.scale, v.z *= a.scale, v.w *= a.scale;
      *reinterpret_cast<float4 *>(qf + rr * D + 4 * c) = v;
    }
  }
  __syncthreads();
  if (a.cos) {
    const int npair = a.rot / 2;
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (npair % 4 == 0 && a.half % 4 == 0 && al16(a.cos) && al16(a.sin)) {
      // Four pairs per item: cos / sin as float4, x0 / x1 as float4 from the
      // staged rows (pairs (i, i + npair), or adjacent when interleaved).
      const int ng = npair / 4;
      constexpr int RI = (128 * (D / 8) + 511) / 512;  // items per thread at most (npair <= D / 2)
      float4 cv[RI], snv[RI];
      bool okv[RI];
      int rv[RI], gv[RI];
#pragma unroll
      for (int u = 0; u < RI; u++) {
        const int e = tid + 512 * u, rr = e / ng, g = e % ng;
        const int64_t pos = past + q0 + rr;
        okv[u] = e < 128 * ng && q0 + rr < a.S && pos < a.CAP;
        rv[u] = rr, gv[u] = g;
        cv[u] = snv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (okv[u]) {
          cv[u] = *reinterpret_cast<const float4 *>(a.cos + pos * a.half + 4 * g);
          snv[u] = *reinterpret_cast<const float4 *>(a.sin + pos * a.half + 4 * g);
        }
      }
#pragma unroll
      for (int u = 0; u < RI; u++) {
        if (!okv[u]) continue;
        float *row = qf + rv[u] * D;
        const float c4[4] = {cv[u].x, cv[u].y, cv[u].z, cv[u].w}, s4[4] = {snv[u].x, snv[u].y, snv[u].z, snv[u].w};
        float x0[4], x1[4];
        if (a.interleaved) {
          const float4 p0 = *reinterpret_cast<const float4 *>(row + 8 * gv[u]);
          const float4 p1 = *reinterpret_cast<const float4 *>(row + 8 * gv[u] + 4);
          x0[0] = p0.x, x1[0] = p0.y, x0[1] = p0.z, x1[1] = p0.w;
          x0[2] = p1.x, x1[2] = p1.y, x0[3] = p1.z, x1[3] = p1.w;
        } else {
          const float4 p0 = *reinterpret_cast<const float4 *>(row + 4 * gv[u]);
          const float4 p1 = *reinterpret_cast<const float4 *>(row + npair + 4 * gv[u]);
          x0[0] = p0.x, x0[1] = p0.y, x0[2] = p0.z, x0[3] = p0.w;
          x1[0] = p1.x, x1[1] = p1.y, x1[2] = p1.z, x1[3] = p1.w;
        }
        float y0[4], y1[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          y0[j] = x0[j] * c4[j] - x1[j] * s4[j];
          y1[j] = x1[j] * c4[j] + x0[j] * s4[j];
        }
        if (a.interleaved) {
          *reinterpret_cast<float4 *>(row + 8 * gv[u]) = make_float4(y0[0], y1[0], y0[1], y1[1]);
          *reinterpret_cast<float4 *>(row + 8 * gv[u] + 4) = make_float4(y0[2], y1[2], y0[3], y1[3]);
        } else {
          *reinterpret_cast<float4 *>(row + 4 * gv[u]) = make_float4(y0[0], y0[1], y0[2], y0[3]);
          *reinterpret_cast<float4 *>(row + npair + 4 * gv[u]) = make_float4(y1[0], y1[1], y1[2], y1[3]);
        }
      }
    } else {
      for (int i = tid; i < 128 * npair; i += 512) {
        const int rr = i / npair, pi = i % npair;
        const int64_t pos = past + q0 + rr;
        if (q0 + rr >= a.S || pos >= a.CAP) continue;
        const float c = a.cos[pos * a.half + pi], sn = a.sin[pos * a.half + pi];
        const int i0 = a.interleaved ? 2 * pi : pi, i1 = a.interleaved ? 2 * pi + 1 : pi + npair;
        const float x0 = qf[rr * D + i0], x1 = qf[rr * D + i1];
        qf[rr * D + i0] = x0 * c - x1 * sn;
        qf[rr * D + i1] = x1 * c + x0 * sn;
      }
    }
  }
  __syncthreads();
  for (int it = tid; it < 128 * (D / 8); it += 512) {
    const int r = it / (D / 8), c = it % (D / 8);
    const float *src = qf + r * D + 8 * c;
    uint4 hv, lv;
    split_bf16x2(src[0], src[1], hv.x, lv.x);
    split_bf16x2(src[2], src[3], hv.y, lv.y);
    split_bf16x2(src[4], src[5], hv.z, lv.z);
    split_bf16x2(src[6], src[7], hv.w, lv.w);
    const uint32_t o = (uint32_t)(c >> 3) * 16384u + sw128_elem(r, (8 * c) & 63);
    *reinterpret_cast<uint4 *>(smem + L::QH + o) = hv;
    *reinterpret_cast<uint4 *>(smem + L::QL + o) = lv;
  }
  __syncthreads();  // the Q staging scratch is consumed before K / V reuse it

  const int nkeys = min(past + a.S, a.CAP);
  const int kend = min(nkeys, past + min(q0 + 128, a.S));  // keys any row of the tile sees
  const float *kc = a.kcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  const float *vc = a.vcache + (int64_t)b * a.kc_bs + (int64_t)kvh * a.kc_hs;
  const uint32_t tmem = *slot;
  const int r = q4 * 32 + lane;
  const int vis = past + q0 + r;  // last key this row sees
  const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
  float m = -INFINITY, l = 0.f;
  float o[DW];
#pragma unroll
  for (int c = 0; c < DW; c++) o[c] = 0.f;
  bool ok = true;
  // Matrix descriptors of the operand planes, formed once; an MMA's operand
  // is its plane's descriptor plus the 16-byte offset of its k slice (the
  // start-address field does not overflow below 256 KB).
  const uint32_t sbase = smem_u32(smem);
  const uint64_t d_qh = sw128_kmajor_desc(sbase + L::QH), d_ql = sw128_kmajor_desc(sbase + L::QL);
  const uint64_t d_kh = sw128_kmajor_desc(sbase + L::KH), d_kl = sw128_kmajor_desc(sbase + L::KL);
  const uint64_t d_vh = sw128_kmajor_desc(sbase + L::VH), d_vl = sw128_kmajor_desc(sbase + L::VL);
  // K / V values of a key tile are loaded into registers two tiles ahead and
  // split into the bf16 planes of the other buffer one tile ahead, while the
  // current tile's Q.K^T runs on the tensor cores.
  constexpr int KI = (64 * (D / 8) + 511) / 512;  // K items (key, 8-dim chunk) per thread
  float kx[KI][8], vx[2][8];
  auto load_tile = [&](int j0) {
#pragma unroll
    for (int i = 0; i < KI; i++) {
      const int e = tid + 512 * i, t = e / (D / 8), c = e % (D / 8);
      if (e < 64 * (D / 8) && j0 + t < kend) {
        const float *src = kc + (int64_t)(j0 + t) * a.kc_rs + 8 * c;
        const float4 u = *reinterpret_cast<const float4 *>(src), w = *reinterpret_cast<const float4 *>(src + 4);
        kx[i][0] = u.x, kx[i][1] = u.y, kx[i][2] = u.z, kx[i][3] = u.w;
        kx[i][4] = w.x, kx[i][5] = w.y, kx[i][6] = w.z, kx[i][7] = w.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) kx[i][j] = 0.f;
      }
    }
    const int pr = tid % 32, g = tid / 32, t0 = 2 * pr;
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const float *src = vc + (int64_t)(j0 + t0 + q) * a.kc_rs + 8 * g;
      if (g < D / 8 && j0 + t0 + q < kend) {
        const float4 u = *reinterpret_cast<const float4 *>(src), w = *reinterpret_cast<const float4 *>(src + 4);
        vx[q][0] = u.x, vx[q][1] = u.y, vx[q][2] = u.z, vx[q][3] = u.w;
        vx[q][4] = w.x, vx[q][5] = w.y, vx[q][6] = w.z, vx[q][7] = w.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) vx[q][j] = 0.f;
      }
    }
  };
  // The registers' tile as bf16 hi / lo planes in buffer `buf`, published to
  // the tensor cores' proxy (the next barrier makes them visible to the
  // issuing thread).
  auto stage_tile = [&](int buf) {
    uint8_t *kb = smem + buf * L::KV_BUF, *vb = smem + buf * L::KV_BUF;
#pragma unroll
    for (int i = 0; i < KI; i++) {
      const int e = tid + 512 * i, t = e / (D / 8), c = e % (D / 8);
      if (e < 64 * (D / 8)) {
        uint4 hv, lv;
        split_bf16x2(kx[i][0], kx[i][1], hv.x, lv.x);
        split_bf16x2(kx[i][2], kx[i][3], hv.y, lv.y);
        split_bf16x2(kx[i][4], kx[i][5], hv.z, lv.z);
        split_bf16x2(kx[i][6], kx[i][7], hv.w, lv.w);
        const uint32_t ob = (uint32_t)(c >> 3) * 8192u + sw128_elem(t, (8 * c) & 63);
        *reinterpret_cast<uint4 *>(kb + L::KH + ob) = hv;
        *reinterpret_cast<uint4 *>(kb + L::KL + ob) = lv;
      }
    }
    // V^T tile: keys 2p, 2p+1 of dims 8g .. 8g+7 as bf16 pairs.
    const int pr = tid % 32, g = tid / 32, t0 = 2 * pr;
    if (g < D / 8) {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        uint32_t hw, lw;
        split_bf16x2(vx[0][j], vx[1][j], hw, lw);
        const uint32_t ov = sw128_elem(8 * g + j, t0);
        *reinterpret_cast<uint32_t *>(vb + L::VH + ov) = hw;
        *reinterpret_cast<uint32_t *>(vb + L::VL + ov) = lw;
      }
    }
    fence_proxy_async_smem();
  };
  // S = Q.K^T of the tile in buffer `buf` (three bf16 products) into TMEM
  // columns 0-63, issued by thread 0.
  auto issue_s = [&](int buf) {
    const uint64_t kvo = (uint64_t)((buf * L::KV_BUF) >> 4);
    constexpr uint32_t idesc_s = umma_idesc(128, 64, 1u, 1u, 1u);
#pragma unroll
    for (int kk = 0; kk < D / 16; kk++) {
      const uint64_t oq = (uint64_t)(((kk >> 2) * 16384u + (kk & 3) * 32u) >> 4);
      const uint64_t ok16 = kvo + (uint64_t)(((kk >> 2) * 8192u + (kk & 3) * 32u) >> 4);
      umma_f16(tmem, d_ql + oq, d_kh + ok16, idesc_s, kk ? 1u : 0u);
      umma_f16(tmem, d_qh + oq, d_kl + ok16, idesc_s, 1u);
      umma_f16(tmem, d_qh + oq, d_kh + ok16, idesc_s, 1u);
    }
    umma_commit(bar_s);
  };
  if (kend > 0) {
    load_tile(0);
    stage_tile(0);
  }
  if (kend > 64) load_tile(64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0 && kend > 0) issue_s(0);
  int it = 0;
  for (int j0 = 0; j0 < kend; j0 += 64, it++) {
    const int buf = it & 1;
    const uint64_t kvo = (uint64_t)((buf * L::KV_BUF) >> 4);
    // While this tile's Q.K^T runs (issued at the end of the previous
    // iteration): the next tile into the other buffer (its last readers, the
    // previous tile's MMAs, have completed), and the loads of the one after.
    if (j0 + 64 < kend) stage_tile(buf ^ 1);
    if (j0 + 128 < kend) load_tile(j0 + 128);
    const bool ok_s = warp_wait_or_abort(bar_s, (uint32_t)(it & 1), abort_flag, a.err);
    tc_fence_after();
    float sv[16];
    float tmax = -INFINITY;
    if (ok_s) {
      uint32_t v[16];
      tmem_ld16(trow + (uint32_t)(cb * 16), v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int t = j0 + cb * 16 + j;
        const float x = (t <= vis && t < kend) ? __uint_as_float(v[j]) : -INFINITY;
        sv[j] = x;
        tmax = fmaxf(tmax, x);
      }
    }
    red_m[cb * 128 + r] = tmax;
    __syncthreads();
    if (*abort_flag) {  // read by every thread after the same barrier: a uniform exit
      ok = false;
      break;
    }
    const float mnew = fmaxf(m, fmaxf(fmaxf(red_m[r], red_m[128 + r]), fmaxf(red_m[256 + r], red_m[384 + r])));
    float psum = 0.f;
    {
      // P = exp(s - max) as bf16 hi / lo, straight into TMEM as the A operand
      // of P.V (keys 2c, 2c+1 in column c): no shared-memory round trip and
      // no proxy fence.
      uint32_t ph[8], pl[8];
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const float e0 = (ok_s && mnew != -INFINITY) ? __expf(sv[j] - mnew) : 0.f;
        const float e1 = (ok_s && mnew != -INFINITY) ? __expf(sv[j + 1] - mnew) : 0.f;
        psum += e0 + e1;
        split_bf16x2(e0, e1, ph[j / 2], pl[j / 2]);
      }
      tmem_st8(trow + L::P_HI + (uint32_t)(cb * 8), ph);
      tmem_st8(trow + L::P_LO + (uint32_t)(cb * 8), pl);
      tmem_st_wait();
    }
    red_l[cb * 128 + r] = psum;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const float corr = m == -INFINITY ? 0.f : __expf(m - mnew);
    l = l * corr + ((red_l[r] + red_l[128 + r]) + (red_l[256 + r] + red_l[384 + r]));
    m = mnew;
    if (tid == 0) {
      if (ok_s) {
        constexpr uint32_t idesc_o = umma_idesc(128, D, 1u, 1u, 1u);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint64_t o16 = kvo + (uint64_t)((kk * 32u) >> 4);
          const uint32_t pc = (uint32_t)(kk * 8);
          umma_f16_ts(tmem + 64, tmem + L::P_LO + pc, d_vh + o16, idesc_o, kk ? 1u : 0u);
          umma_f16_ts(tmem + 64, tmem + L::P_HI + pc, d_vl + o16, idesc_o, 1u);
          umma_f16_ts(tmem + 64, tmem + L::P_HI + pc, d_vh + o16, idesc_o, 1u);
        }
      }
      umma_commit(bar_o);  // also when skipped, so every wait ends
      // The next tile's Q.K^T right behind it: its K planes were staged and
      // fenced before this tile's two barriers, S has been read, and P sits in
      // other TMEM columns. It runs under the output update below.
      if (j0 + 64 < kend) issue_s(buf ^ 1);
    }
    const bool ok_o = warp_wait_or_abort(bar_o, (uint32_t)(it & 1), abort_flag, a.err) && ok_s;
    tc_fence_after();
    if (ok_o) {
#pragma unroll
      for (int c0 = 0; c0 < DW; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(trow + 64u + (uint32_t)(cb * DW + c0), v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; j++) o[c0 + j] = fmaf(o[c0 + j], corr, __uint_as_float(v[j]));
      }
    }
    // No barrier here: the next tile's S issue needs its K / V planes, which
    // every thread staged (and fenced) before this tile's two barriers; the
    // P.V that read P and V has completed for every thread that goes on.
  }
  if (ok && q0 + r < a.S) {
    const float inv = 1.f / l;
    const int64_t off = (int64_t)(b * a.S + q0 + r) * a.H * D + h * D + cb * DW;
#pragma unroll
    for (int c = 0; c < DW; c += 4) {
      const float4 v4 = make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
      if (a.out) *reinterpret_cast<float4 *>(a.out + off + c) = v4;
      if (a.out16) store_f16x4(a.out16 + off + c, v4);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

__global__ void advance_kernel(int32_t *past, int n, int delta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) past[i] += delta;
}

unsigned grid_for(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 16));
}

}  // namespace

void launch_rmsnorm(const float *x, const float *skip, const float *gamma, float *y, float *sum_out, int64_t rows,
                    int D, double eps, int64_t per, int64_t gstride, cudaStream_t s, int64_t gamma_rs, __half *y16) {
  if (rows <= 0) return;
  if (launch_norm_rows_cta<false>(x, skip, gamma, nullptr, y, sum_out, rows, D, eps, per, gstride, gamma_rs, s, y16))
    return;
  B2M_REQUIRE(y, B2M_ERR_INVALID_ARGUMENT,
              "RMSNorm f16: y may be NULL only for rows of d % 4 == 0 floats with 16-byte aligned operands");
  if (y16) {  // the fallback kernels write fp32 only: round the rows after them
    launch_rmsnorm(x, skip, gamma, y, sum_out, rows, D, eps, per, gstride, s, gamma_rs, nullptr);
    b2m::launch_f32_to_f16(y, y16, rows, D, D, 0, s);
    return;
  }
  const unsigned g = (unsigned)((rows + 7) / 8);
  const int vpl = (D + 31) / 32;
#define B2M_RMS(V) \
  rmsnorm_kernel<V><<<g, 256, 0, s>>>(x, skip, gamma, y, sum_out, rows, D, eps, per, gstride, gamma_rs)
  if (vpl <= 4) B2M_RMS(4);
  else if (vpl <= 8) B2M_RMS(8);
  else if (vpl <= 16) B2M_RMS(16);
  else if (vpl <= 24) B2M_RMS(24);
  else if (vpl <= 32) B2M_RMS(32);
  else if (vpl <= 64) B2M_RMS(64);
  else rmsnorm_long_kernel<<<g, 256, 0, s>>>(x, skip, gamma, y, sum_out, rows, D, eps, per, gstride, gamma_rs);
#undef B2M_RMS
  B2M_CUDA(cudaGetLastError());
}

void launch_layernorm(const float *x, const float *skip, const float *gamma, const float *beta, float *y,
                      float *sum_out, int64_t rows, int D, double eps, cudaStream_t s, __nv_bfloat16 *p0,
                      __nv_bfloat16 *p1) {
  if (rows <= 0) return;
  if (launch_norm_rows_cta<true>(x, skip, gamma, beta, y, sum_out, rows, D, eps, rows, 0, 0, s, nullptr, p0, p1))
    return;
  if (p0) {  // the fallback kernels write fp32 only: split the rows after them
    launch_layernorm(x, skip, gamma, beta, y, sum_out, rows, D, eps, s, nullptr, nullptr);
    ::launch_f32_split(y, D, p0, p1, rows, D, D, s);
    return;
  }
  const unsigned g = (unsigned)((rows + 7) / 8);
  const int vpl = (D + 31) / 32;
#define B2M_LN(V) layernorm_kernel<V><<<g, 256, 0, s>>>(x, skip, gamma, beta, y, sum_out, rows, D, eps)
  if (vpl <= 4) B2M_LN(4);
  else if (vpl <= 8) B2M_LN(8);
  else if (vpl <= 16) B2M_LN(16);
  else if (vpl <= 24) B2M_LN(24);
  else if (vpl <= 32) B2M_LN(32);
  else if (vpl <= 64) B2M_LN(64);
  else layernorm_long_kernel<<<g, 256, 0, s>>>(x, skip, gamma, beta, y, sum_out, rows, D, eps);
#undef B2M_LN
  B2M_CUDA(cudaGetLastError());
}

void launch_silu_mul(const float *gate, const float *up, int64_t g_rs, int64_t u_rs, float *y, int64_t rows,
                     int64_t D, cudaStream_t s, __half *y16) {
  if (rows * D <= 0) return;
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = D % 4 == 0 && g_rs % 4 == 0 && u_rs % 4 == 0 && al(gate) && al(up) && al(y) &&
                   (reinterpret_cast<uintptr_t>(y16) & 7) == 0;
  if (y16 && !vec) {  // the scalar path writes fp32 only: round the rows after it
    launch_silu_mul(gate, up, g_rs, u_rs, y, rows, D, s, nullptr);
    b2m::launch_f32_to_f16(y, y16, rows, D, D, 0, s);
    return;
  }
  const int64_t cols = vec ? D / 4 : D;
  const dim3 grid((unsigned)std::min<int64_t>((cols + 255) / 256, 64), (unsigned)std::min<int64_t>(rows, 65535));
  if (vec) silu_mul_kernel<true><<<grid, 256, 0, s>>>(gate, up, g_rs, u_rs, y, rows, D, y16);
  else silu_mul_kernel<false><<<grid, 256, 0, s>>>(gate, up, g_rs, u_rs, y, rows, D, nullptr);
  B2M_CUDA(cudaGetLastError());
}

void launch_silu_mul_tiles(const float *y, int64_t rows, int64_t I, float *act, __half *act16, cudaStream_t s) {
  if (rows * I <= 0) return;
  silu_mul_tiles_kernel<<<grid_for(rows * (I / 4), 256), 256, 0, s>>>(y, rows, I, act, act16);
  B2M_CUDA(cudaGetLastError());
}

void launch_gelu(const float *x, float *y, int64_t n, cudaStream_t s) {
  if (n <= 0) return;
  gelu_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, y, n);
  B2M_CUDA(cudaGetLastError());
}

void launch_gelu_split(const float *x, float *y, __nv_bfloat16 *p0, __nv_bfloat16 *p1, int64_t n, cudaStream_t s) {
  if (n <= 0) return;
  gelu_split_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(x, y, p0, p1, n / 4);
  B2M_CUDA(cudaGetLastError());
}

void launch_add(const float *a, const float *b, float *y, int64_t rows, int64_t D, int b_bcast, cudaStream_t s) {
  if (rows * D <= 0) return;
  add_kernel<<<grid_for(rows * D, 256), 256, 0, s>>>(a, b, y, rows, D, b_bcast);
  B2M_CUDA(cudaGetLastError());
}

void launch_gather_rows(const float *table, const int64_t *ids, float *y, int64_t rows, int64_t V, int64_t D,
                        int32_t *err, cudaStream_t s) {
  if (rows <= 0) return;
  gather_rows_kernel<<<(unsigned)rows, 256, 0, s>>>(table, ids, y, rows, V, D, err);
  B2M_CUDA(cudaGetLastError());
}

int argmax_chunks(int64_t rows, int64_t V) {
  const int64_t want = (4 * (int64_t)b2m::device_sm_count() + rows - 1) / std::max<int64_t>(rows, 1);
  const int64_t by_len = (V + 4095) / 4096;
  return (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(want, by_len), 1024));
}

void launch_argmax(const float *x, int64_t *out, int64_t rows, int64_t V, float *pv, int64_t *pi, cudaStream_t s) {
  if (rows <= 0) return;
  const int nchunk = argmax_chunks(rows, V);
  const int64_t chunk = ((V + nchunk - 1) / nchunk + 3) / 4 * 4;
  argmax_partial_kernel<<<dim3((unsigned)nchunk, (unsigned)rows), 256, 0, s>>>(x, V, chunk, pv, pi);
  B2M_CUDA(cudaGetLastError());
  argmax_final_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(pv, pi, nchunk, out, rows, V);
  B2M_CUDA(cudaGetLastError());
}

// Runs the attention proper (keys already in place) for the addressing in
// `a`: the single-token decode kernel for cached causal calls of one query,
// the tiled kernel for head dims 32..128 in steps of 32, the per-query-warp
// kernel otherwise.
static bool decode_shape(const GqaArgs &a) {
  const int D = a.D, G = a.H / a.KVH;
  const bool dok = D == 32 || D == 64 || D == 96 || D == 128;
  return a.S == 1 && a.past && a.causal && !a.mask && dok && (G == 1 || G == 2 || G == 4 || G == 8);
}

// The tensor-core kernel: MultiHeadAttention (keys from the projected rows)
// of head_dim 64 with at most 128 queries and keys, 16-byte aligned rows.
static bool mha_tc_shape(const GqaArgs &a) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return !a.past && a.D == 64 && a.S >= 1 && a.S <= 128 && a.kv_len >= 1 && a.kv_len <= 128 && a.q_rs % 4 == 0 &&
         a.kc_rs % 4 == 0 && a.kc_bs % 4 == 0 && a.kc_hs % 4 == 0 && al(a.q) && al(a.kcache) && al(a.vcache);
}

// The tensor-core flash kernel: causal GroupQueryAttention over the KV cache
// (prefill or chunked prefill, more than one query), head_dim 64 or 128,
// 16-byte aligned rows, no additive bias.
static bool fa_tc_shape(const GqaArgs &a) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return a.past && a.causal && !a.mask && (a.D == 64 || a.D == 128) && a.S >= 2 && a.H % a.KVH == 0 &&
         a.q_rs % 4 == 0 && a.kc_rs % 4 == 0 && a.kc_bs % 4 == 0 && a.kc_hs % 4 == 0 && (int64_t)a.H * a.D % 4 == 0 &&
         al(a.q) && al(a.kcache) && al(a.vcache) && al(a.out) && (a.rot == 0 || !a.cos || a.rot <= a.D);
}

static void launch_attend(const GqaArgs &a, float *split_part, int nsplit, bool exact, uint32_t *counters,
                          cudaStream_t s) {
  const int D = a.D, G = a.H / a.KVH;
  const bool dok = D == 32 || D == 64 || D == 96 || D == 128;
  bool wrote16 = false, wrote_planes = false;  // the kernel wrote a.out16 / a.p0, a.p1 itself
  if (decode_shape(a)) {
    if (!split_part) nsplit = 1;
    dim3 grid((unsigned)a.KVH, (unsigned)a.B, (unsigned)nsplit);
    const int64_t slots = (int64_t)a.B * a.H * nsplit;
    float *pm = split_part, *pl = pm ? pm + slots : nullptr, *po = pm ? pl + slots : nullptr;
#define B2M_DEC(DD, GG) \
  if (D == DD && G == GG) gqa_decode_kernel<DD, GG><<<grid, 256, 0, s>>>(a, pm, pl, po, nsplit > 1 ? counters : nullptr);
    B2M_DEC(32, 1) B2M_DEC(32, 2) B2M_DEC(32, 4) B2M_DEC(32, 8)
    B2M_DEC(64, 1) B2M_DEC(64, 2) B2M_DEC(64, 4) B2M_DEC(64, 8)
    B2M_DEC(96, 1) B2M_DEC(96, 2) B2M_DEC(96, 4) B2M_DEC(96, 8)
    B2M_DEC(128, 1) B2M_DEC(128, 2) B2M_DEC(128, 4) B2M_DEC(128, 8)
#undef B2M_DEC
    B2M_CUDA(cudaGetLastError());
    if (nsplit > 1 && !counters) {
      gqa_decode_combine_kernel<<<dim3((unsigned)a.H, (unsigned)a.B), 128, 0, s>>>(pm, pl, po, a.out, a.H, D, nsplit);
    } else {
      wrote16 = true;
    }
  } else if (!exact && fa_tc_shape(a)) {
    wrote16 = true;
    if (D == 128) {
      b2m::set_smem_limit_once<fa_tc_kernel<128>>((int)FaLayout<128>::BYTES);
      fa_tc_kernel<128><<<dim3((unsigned)((a.S + 127) / 128), (unsigned)a.H, (unsigned)a.B), 512,
                          FaLayout<128>::BYTES, s>>>(a);
    } else {
      b2m::set_smem_limit_once<fa_tc_kernel<64>>((int)FaLayout<64>::BYTES);
      fa_tc_kernel<64><<<dim3((unsigned)((a.S + 127) / 128), (unsigned)a.H, (unsigned)a.B), 512,
                         FaLayout<64>::BYTES, s>>>(a);
    }
  } else if (!exact && mha_tc_shape(a)) {
    wrote_planes = true;
    b2m::set_smem_limit_once<mha_tc_kernel>((int)MTC_BYTES);
    mha_tc_kernel<<<dim3((unsigned)a.H, (unsigned)a.B), 512, MTC_BYTES, s>>>(a);
  } else if (dok) {
    dim3 grid((unsigned)((a.S + 63) / 64), (unsigned)a.H, (unsigned)a.B);
    const int smem = (2 * D * 68 + 64 * D + 64 * 68) * 4;
    switch (D) {
      case 32:
        b2m::set_smem_limit_once<gqa_prefill_kernel<32>>(smem);
        gqa_prefill_kernel<32><<<grid, 256, smem, s>>>(a);
        break;
      case 64:
        b2m::set_smem_limit_once<gqa_prefill_kernel<64>>(smem);
        gqa_prefill_kernel<64><<<grid, 256, smem, s>>>(a);
        break;
      case 96:
        b2m::set_smem_limit_once<gqa_prefill_kernel<96>>(smem);
        gqa_prefill_kernel<96><<<grid, 256, smem, s>>>(a);
        break;
      default:
        b2m::set_smem_limit_once<gqa_prefill_kernel<128>>(smem);
        gqa_prefill_kernel<128><<<grid, 256, smem, s>>>(a);
        break;
    }
  } else {
    dim3 grid((unsigned)((a.S + 7) / 8), (unsigned)a.H, (unsigned)a.B);
    gqa_attend_kernel<<<grid, 256, 0, s>>>(a);
  }
  B2M_CUDA(cudaGetLastError());
  if (a.out16 && !wrote16)  // the other kernels write fp32 only: round after them
    b2m::launch_f32_to_f16(a.out, a.out16, (int64_t)a.B * a.S, (int64_t)a.H * D, (int64_t)a.H * D, 0, s);
  if (a.p0 && !wrote_planes)
    ::launch_f32_split(a.out, (int64_t)a.H * D, a.p0, a.p1, (int64_t)a.B * a.S, (int64_t)a.H * D, (int64_t)a.H * D, s);
}

// Whether launch_gqa's attention kernel for these arguments writes the f16
// output itself (the decode kernel when its key splits merge in the kernel,
// the flash prefill kernel), so that the fp32 output may be omitted.
bool gqa_writes_f16(const float *q, int64_t q_rs, const float *kcache, const float *vcache, const int32_t *past,
                    const float *cos, int rot, int B, int S, int H, int KVH, int D, int CAP, int nsplit, bool exact,
                    bool counters) {
  GqaArgs a{q, nullptr, nullptr, q_rs, 0, const_cast<float *>(kcache), const_cast<float *>(vcache), past, cos,
            nullptr, 0, rot, 0, nullptr, B, S, H, KVH, D, CAP, 1.f, nullptr};
  a.kc_rs = D;
  a.kc_hs = (int64_t)CAP * D;
  a.kc_bs = (int64_t)KVH * CAP * D;
  a.causal = 1;
  a.kv_len = CAP;
  a.mask = nullptr;
  a.mask_bs = a.mask_hs = a.mask_qs = 0;
  if (decode_shape(a)) return nsplit <= 1 || counters;
  return !exact && fa_tc_shape(a);
}

// Key splits of the decode kernel: enough CTAs for two per SM, at least 128
// cache positions per split. Partial-state floats: B*H*nsplit*(2 + D).
int gqa_decode_splits(int B, int S, int H, int KVH, int D, int CAP) {
  if (S != 1 || B * KVH <= 0) return 1;
  const int want = (2 * b2m::device_sm_count() + B * KVH - 1) / (B * KVH);
  return std::max(1, std::min(want, (CAP + 127) / 128));
}

void launch_gqa(const float *q, const float *k, const float *v, int64_t q_rs, int64_t kv_rs, float *kcache,
                float *vcache, const int32_t *past, const float *cos, const float *sin, int half, int rot,
                int interleaved, float *out, int B, int S, int H, int KVH, int D, int CAP, float scale, int32_t *err,
                float *split_part, int nsplit, bool exact, uint32_t *counters, cudaStream_t s, __half *out16,
                const float *qk_gain, double qk_eps) {
  GqaArgs a{q, k, v, q_rs, kv_rs, kcache, vcache, past, cos, sin, half, rot, interleaved, out,
            B, S, H, KVH, D, CAP, scale, err};
  a.out16 = out16;
  a.kc_rs = D;
  a.kc_hs = (int64_t)CAP * D;
  a.kc_bs = (int64_t)KVH * CAP * D;
  a.causal = 1;
  a.kv_len = CAP;
  a.mask = nullptr;
  a.mask_bs = a.mask_hs = a.mask_qs = 0;
  if (qk_gain) {
    // Folded where the head-rows norm would take its float4 form (the
    // arithmetic the kernels reproduce): the decode kernel normalises q and
    // k in its prologue and appends; for the flash prefill kernel the append
    // kernel normalises k and the flash kernel q.
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool f4 = D % 4 == 0 && D <= 128 && q_rs % 4 == 0 && kv_rs % 4 == 0 && al(q) && al(k) && al(v) &&
                    al(qk_gain);
    if (f4 && decode_shape(a)) {
      a.qk_gain = qk_gain;
      a.qk_eps = qk_eps;
      launch_attend(a, split_part, nsplit, exact, counters, s);
      return;
    }
    if (f4 && !exact && fa_tc_shape(a)) {
      a.qk_gain = qk_gain;
      a.qk_eps = qk_eps;
      const int64_t items = (int64_t)B * S * KVH;
      gqa_append_kernel<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(a);
      B2M_CUDA(cudaGetLastError());
      launch_attend(a, split_part, nsplit, exact, counters, s);
      return;
    }
    float *qw = const_cast<float *>(q), *kw = const_cast<float *>(k);
    if (k == q + (int64_t)H * D && kv_rs == q_rs) {  // q and k heads adjacent in the rows: one launch
      launch_rmsnorm(qw, nullptr, qk_gain, qw, nullptr, (int64_t)B * S * (H + KVH), D, qk_eps, H + KVH, q_rs, s, D);
    } else {
      launch_rmsnorm(qw, nullptr, qk_gain, qw, nullptr, (int64_t)B * S * H, D, qk_eps, H, q_rs, s, D);
      launch_rmsnorm(kw, nullptr, qk_gain + (int64_t)H * D, kw, nullptr, (int64_t)B * S * KVH, D, qk_eps, KVH, kv_rs,
                     s, D);
    }
  }
  const int64_t items = (int64_t)B * S * KVH;
  gqa_append_kernel<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(a);
  B2M_CUDA(cudaGetLastError());
  launch_attend(a, split_part, nsplit, exact, counters, s);
}

void launch_mha(const float *q, const float *k, const float *v, int64_t q_rs, int64_t kv_rs, const float *mask,
                int64_t mask_bs, int64_t mask_hs, int64_t mask_qs, float *out, int B, int S, int T, int H, int KVH,
                int D, float scale, int causal, int32_t *err, bool exact, cudaStream_t s, __nv_bfloat16 *planes) {
  GqaArgs a{q, k, v, q_rs, kv_rs, const_cast<float *>(k), const_cast<float *>(v), nullptr, nullptr, nullptr, 0, 0,
            0, out, B, S, H, KVH, D, T, scale, err};
  if (planes) {
    a.p0 = planes;
    a.p1 = planes + (int64_t)B * S * H * D;
  }
  a.kc_rs = kv_rs;
  a.kc_hs = D;
  a.kc_bs = (int64_t)T * kv_rs;
  a.causal = causal;
  a.kv_len = T;
  a.mask = mask;
  a.mask_bs = mask_bs;
  a.mask_hs = mask_hs;
  a.mask_qs = mask_qs;
  launch_attend(a, nullptr, 1, exact, nullptr, s);
}

void launch_rotary(const float *x, int64_t x_rs, const int64_t *pos, int pos_per_batch, const float *cos,
                   const float *sin, int half, int max_pos, float *y, int64_t y_rs, int B, int S, int heads, int D,
                   int rot, int interleaved, int32_t *err, cudaStream_t s) {
  const int64_t items = (int64_t)B * S * heads;
  if (items == 0) return;
  rotary_kernel<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(x, x_rs, pos, pos_per_batch, cos, sin, half, max_pos, y,
                                                            y_rs, B, S, heads, D, rot, interleaved, err);
  B2M_CUDA(cudaGetLastError());
}

void launch_advance_positions(int32_t *past, int n, int delta, cudaStream_t s) {
  if (n <= 0) return;
  advance_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(past, n, delta);
  B2M_CUDA(cudaGetLastError());
}
