// DynamicQuantizeLinear on the device (opDynamicQuantizeLinear,
// lib/src/onnx_ops.dart:3556-3583), bit-exact:
//   mn = min(0, min x), mx = max(0, max x)       (NaN ignored, as `v < mn`)
//   scale = f32((double)mx - (double)mn) / 255)    (double, then stored f32)
//   zp = roundEven(clamp(f32(-mn / scale), 0, 255)), 0 when scale == 0
//   y = clamp(roundEven(f32(x / scale)) + zp, 0, 255), zp when scale == 0
// f32(x / scale) computed in double equals the correctly rounded fp32
// quotient (double carries more than 2 * 24 + 2 bits, so the second rounding
// is innocuous); the kernel uses the fp32 division directly.
//
// Two launches: a grid-wide min/max whose last block derives scale and zero
// point into device memory, then the elementwise quantization, which reads
// them there (so a chain into MatMulInteger never leaves the device).
#include <algorithm>

#include "b2m_internal.cuh"
#include "tc_common.cuh"

namespace {

constexpr int DQ_THREADS = 256;

__device__ __forceinline__ int64_t round_even_ll(float v) { return __float2ll_rn(v); }

// partial[2 * block] = (min, max) of the block's elements (starting from 0);
// the last block to finish reduces all partials and writes scale / zp.
__global__ void __launch_bounds__(DQ_THREADS) dql_range_kernel(const float *__restrict__ x, int64_t n, float *partial,
                                                               unsigned int *done, float *scale_out, uint8_t *zp_out) {
  float mn = 0.f, mx = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * DQ_THREADS + threadIdx.x; i < n; i += (int64_t)gridDim.x * DQ_THREADS) {
    const float v = x[i];
    mn = v < mn ? v : mn;
    mx = v > mx ? v : mx;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float a = __shfl_xor_sync(0xffffffffu, mn, off), b = __shfl_xor_sync(0xffffffffu, mx, off);
    mn = a < mn ? a : mn;
    mx = b > mx ? b : mx;
  }
  __shared__ float smn[DQ_THREADS / 32], smx[DQ_THREADS / 32];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    smn[warp] = mn;
    smx[warp] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < DQ_THREADS / 32; w++) {
      mn = smn[w] < mn ? smn[w] : mn;
      mx = smx[w] > mx ? smx[w] : mx;
    }
    partial[2 * blockIdx.x] = mn;
    partial[2 * blockIdx.x + 1] = mx;
    __threadfence();
    last = atomicAdd(done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  const volatile float *vp = partial;
  mn = 0.f;
  mx = 0.f;
  for (unsigned b = 0; b < gridDim.x; b++) {
    const float a = vp[2 * b], c = vp[2 * b + 1];
    mn = a < mn ? a : mn;
    mx = c > mx ? c : mx;
  }
  *done = 0;  // ready for the next call without a memset
  const float scale = (float)(((double)mx - (double)mn) / 255.0);
  int64_t zp = 0;
  if (scale != 0.f) {
    double zf = (double)(float)(-(double)mn / (double)scale);
    zf = zf < 0.0 ? 0.0 : (zf > 255.0 ? 255.0 : zf);
    zp = __double2ll_rn(zf);
  }
  *scale_out = scale;
  *zp_out = (uint8_t)zp;
}

__global__ void __launch_bounds__(DQ_THREADS) dql_quantize_kernel(const float *__restrict__ x, int64_t n,
                                                                  const float *scale_p, const uint8_t *zp_p,
                                                                  uint8_t *__restrict__ y) {
  const float scale = *scale_p;
  const int64_t zp = *zp_p;
  const int64_t stride = (int64_t)gridDim.x * DQ_THREADS * 4;
  for (int64_t i0 = ((int64_t)blockIdx.x * DQ_THREADS + threadIdx.x) * 4; i0 < n; i0 += stride) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int64_t i = i0 + j;
      if (i >= n) break;
      int64_t q = zp;
      if (scale != 0.f) q = round_even_ll(__fdiv_rn(x[i], scale)) + zp;
      y[i] = (uint8_t)(q < 0 ? 0 : (q > 255 ? 255 : q));
    }
  }
}

}  // namespace

constexpr int DQ_MAX_BLOCKS = 1024;

size_t dql_partial_floats() { return 2 * DQ_MAX_BLOCKS; }

void launch_dynamic_quantize(const float *x, int64_t n, uint8_t *y, float *scale, uint8_t *zp, float *partial,
                             uint32_t *counter, cudaStream_t s) {
  const int sms = b2m::device_sm_count();
  const int64_t want = (n + DQ_THREADS * 8 - 1) / (DQ_THREADS * 8);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(want, std::min(sms * 4, DQ_MAX_BLOCKS)));
  dql_range_kernel<<<blocks, DQ_THREADS, 0, s>>>(x, n, partial, counter, scale, zp);
  B2M_CUDA(cudaGetLastError());
  if (n > 0) {
    const int64_t qwant = (n + DQ_THREADS * 4 - 1) / (DQ_THREADS * 4);
    const int qblocks = (int)std::max<int64_t>(1, std::min<int64_t>(qwant, (int64_t)sms * 16));
    dql_quantize_kernel<<<qblocks, DQ_THREADS, 0, s>>>(x, n, scale, zp, y);
    B2M_CUDA(cudaGetLastError());
  }
}
